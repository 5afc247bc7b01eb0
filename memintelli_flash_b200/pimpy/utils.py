"""Metrics and the dense slice-pair contraction helper of ``memintelli.pimpy.utils``.

``SNR``/``RE``/``ABSE`` follow memintelli/pimpy/utils.py:32-41; ``dot_high_dim``
is the einsum of memintelli/pimpy/utils.py:11-29, kept for API compatibility
(the engine never materialises this tensor).
"""
import numpy as np
import torch


def dot_high_dim(x, y):
    if len(x.shape) == 5:
        return torch.einsum("nmijk, mpskl->nmpisjl", x, y)
    elif len(x.shape) == 6:
        return torch.einsum("bnmijk, mpskl->bnmpisjl", x, y)
    raise ValueError('The input data dimension is not supported!')


def ABSE(ytest, ypred):
    return np.sum(np.abs((ytest - ypred) / ytest)) / (ytest.shape[0] * ytest.shape[1])


def SNR(ytest, ypred):
    return 10 * np.log10(np.sum(ytest ** 2) / np.sum((ytest - ypred) ** 2))


def RE(ytest, ypred):
    return np.sqrt(np.sum((ytest - ypred) ** 2)) / np.sqrt(np.sum(ytest ** 2))
