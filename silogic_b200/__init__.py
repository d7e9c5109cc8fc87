"""silogic_b200 -- differentiable logic-gate networks on NVIDIA B200 (sm_100a).

A from-scratch CUDA implementation of the logic-gate-network hot path behind the
module API of the ``silogic`` library: ``LogicLayer``, ``LogicNet``,
``ConvLogicTree``, ``OrPool``, ``LogicTreeNet``, ``WARPLayer``, ``LUTkLayer``, ...
Soft forward/backward and the bit-packed hard circuit run in hand-written
kernels (``libsilogic_b200.so``, C ABI in ``include/silogic_b200.h``); there is
no CPU implementation and no Triton.
"""
__version__ = "0.1.0"

from .functional import (BASIS_COEFFS, TRUTH_TABLES, ste_threshold, sign_ste, ternary_ste,
                         binarize_ste, gate_probs, residual_logit)
from .connectomes import build_connectome
from .nodes import build_node, NODES, RELAXATIONS
from .heads import GroupSum, build_decoder, LearnedDecoder
from .layers import (LogicLayer, WARPLayer, WARPLayerN, LUTkLayer, LUTNodeLayer,
                     ConvLogicTree, ConvLogicLayer, OrPool)
from .models import (LogicNet, WARPNet, WARPNetN, LUTkNet, LUTNodeNet, LogicConvNet,
                     LogicTreeNet)
from .encoders import LearnedThermometerEncoder
from .data import (binarize_spatial, MNIST_THRESH, SEVEN_THRESH, FOUR_THRESH, FIVE_THRESH,
                   CIFAR3_THRESH, EDGE_THRESH)

__all__ = [
    "BASIS_COEFFS", "TRUTH_TABLES", "ste_threshold", "sign_ste", "ternary_ste",
    "binarize_ste", "gate_probs", "residual_logit",
    "build_connectome", "build_node", "NODES", "RELAXATIONS",
    "GroupSum", "build_decoder", "LearnedDecoder",
    "LogicLayer", "WARPLayer", "WARPLayerN", "LUTkLayer", "LUTNodeLayer",
    "ConvLogicTree", "ConvLogicLayer", "OrPool",
    "LogicNet", "WARPNet", "WARPNetN", "LUTkNet", "LUTNodeNet", "LogicConvNet", "LogicTreeNet",
    "LearnedThermometerEncoder",
    "binarize_spatial", "MNIST_THRESH", "SEVEN_THRESH", "FOUR_THRESH", "FIVE_THRESH",
    "CIFAR3_THRESH", "EDGE_THRESH",
]
