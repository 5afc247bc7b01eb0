"""B200 counterparts of ``memintelli.NN_layers`` (LinearMem, Conv2dMem)."""
from .linear import LinearMem
from .convolution import Conv2dMem
from .functions import linear_mem_func, conv2d_mem_func, LinearMemRunc, Conv2dMemRunc

__all__ = ['LinearMem', 'Conv2dMem', 'linear_mem_func', 'conv2d_mem_func', 'LinearMemRunc', 'Conv2dMemRunc']
