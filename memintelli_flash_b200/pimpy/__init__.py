"""B200 counterpart of ``memintelli.pimpy`` (memintelli/pimpy/__init__.py:5)."""
__all__ = ['SlicedData', 'DPETensor', 'RE', 'ABSE', 'SNR', 'dot_high_dim']
__version__ = '0.1.1'

from .data_formats import SlicedData
from .memmat_tensor import DPETensor
from .utils import RE, ABSE, SNR, dot_high_dim
