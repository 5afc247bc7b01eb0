"""memintelli_flash_b200: B200 (sm_100a) kernels for Memintelli's CIM bit-sliced matmul.

Drop-in for the hot path of the reference package:
``memintelli.pimpy`` (SlicedData, DPETensor, SNR/RE/ABSE, dot_high_dim) and
``memintelli.NN_layers`` (LinearMem, Conv2dMem).
"""
from . import pimpy, NN_layers
from .pimpy import SlicedData, DPETensor, SNR, RE, ABSE, dot_high_dim
from .NN_layers import LinearMem, Conv2dMem

__version__ = "0.1.0"
