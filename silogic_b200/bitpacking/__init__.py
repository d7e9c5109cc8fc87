"""Bit-packed inference (API of ``silogic.bitpacking``), GPU-resident.

64 samples per int64 word, one CUDA launch per FC layer / per conv block (OR-pool
fused), popcount GroupSum on the device.
"""
import numpy as np
import torch

from .. import _hard
from .plan import HardPlan, HardGraph
from .convert import convert_logic_net, convert_logic_conv_net, convert_layer, convert_head
from .artifact import save_packed, load_packed
from .benchmark import (BenchResult, run_benchmark, run_conv_benchmark, print_report,
                        speedup_summary)
from .packed import (BitpackedNet, BitpackedConvNet, BitpackedConvGPUNet, BitpackedGPULayer,
                     BitpackedConvGPULayer, packed_unfold_gpu, packed_or_pool_gpu,
                     PackedGroupSumHead, PackedLearnedHead)

# reference names of the bit-packed heads (packed_layer.py:545-605)
BitpackedGroupSumHead = PackedGroupSumHead
BitpackedLearnedHead = PackedLearnedHead

# GPU bit-packed kernels are available (name kept from the reference; no Triton is used).
HAS_TRITON = True


def n_words(B):
    """Number of 64-bit words for ``B`` samples."""
    return _hard.n_words(B)


def pack_bits(x):
    """``[B, dim]`` -> ``[dim, ceil(B/64)]`` int64 (numpy in -> numpy out, via the GPU)."""
    was_np = isinstance(x, np.ndarray)
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda() if was_np else x
    B = t.shape[0]
    p = _hard.pack(t)[:, :n_words(B)]
    return p.cpu().numpy() if was_np else p


def unpack_bits(packed, B):
    """``[dim, n_words]`` int64 -> ``[B, dim]`` uint8."""
    was_np = isinstance(packed, np.ndarray)
    t = torch.from_numpy(np.ascontiguousarray(packed)).cuda() if was_np else packed
    if t.shape[-1] % 2:
        t = torch.nn.functional.pad(t, (0, 1))
    out = _hard.unpack(t.contiguous(), B)
    return out.cpu().numpy() if was_np else out


__all__ = ["convert_logic_net", "convert_logic_conv_net", "convert_layer", "convert_head",
           "BitpackedNet", "BitpackedConvNet", "BitpackedConvGPUNet", "BitpackedGPULayer",
           "BitpackedConvGPULayer", "packed_unfold_gpu", "packed_or_pool_gpu",
           "pack_bits", "unpack_bits", "n_words", "HAS_TRITON", "BitpackedGroupSumHead",
           "BitpackedLearnedHead", "HardPlan", "HardGraph", "run_benchmark",
           "run_conv_benchmark", "print_report", "speedup_summary", "BenchResult",
           "save_packed", "load_packed"]
