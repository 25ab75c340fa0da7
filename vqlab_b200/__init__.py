"""B200-native VQ expert runtime: VQSwitchLinear / VQLinear over vq_pack codes.

The compute is libvqb200.so (hand-written sm_100a CUDA behind the C ABI in
include/vqb.h); this package is the PyTorch-facing mirror of the reference
modules src/vqlab/runtime/vq_switch.py and vq_dense.py.
"""
from . import vq_pack
from .artifact import load_vq_layers
from .vq_dense import VQLinear
from .vq_switch import VQSwitchLinear, skipzero_row_table

__all__ = ["VQSwitchLinear", "VQLinear", "vq_pack", "load_vq_layers", "skipzero_row_table"]
