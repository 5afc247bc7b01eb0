"""``Conv2dMem``: CIM 2-D convolution without im2col (memintelli/NN_layers/convolution.py:52-140).

The reference unfolds the input with ``F.unfold`` (K order c*kh*kw + i*kw + j),
slices the (N, L, K) tensor, multiplies and folds back to NCHW.  Here the
slicing kernel gathers the unfolded elements straight from the NCHW input and
the MVM kernel stores its rows directly in NCHW order with the bias fused, so
neither the unfolded fp32 tensor nor the (N, L, Cout) result is materialised.
"""
import math

import torch
import torch.nn as nn

from .. import _native as N
from ..pimpy.data_formats import SlicedData
from .functions import conv2d_mem_func


def _pair(x):
    if isinstance(x, tuple):
        assert len(x) == 2
        return x
    if isinstance(x, int):
        return (x, x)
    raise ValueError("x must be x tuple or int")


class Conv2dMem(nn.Module):
    def __init__(self, engine, in_channels, out_channels, kernel_size, input_slice, weight_slice, stride=1,
                 padding=0, dilation=1, bias=True, device=None, dtype=None, bw_e=None, input_paral_size=(1, 32),
                 weight_paral_size=(32, 32), input_quant_gran=(1, 32), weight_quant_gran=(32, 32)):
        super().__init__()
        factory_kwargs = {'device': device, 'dtype': dtype}
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = kernel_size
        self.stride = stride
        self.padding = padding
        self.dilation = dilation
        self.weight = nn.Parameter(torch.empty((out_channels, in_channels, kernel_size, kernel_size),
                                               **factory_kwargs))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_channels, **factory_kwargs))
        else:
            self.register_parameter('bias', None)
        self.reset_parameters()
        self.weight_slice_method = torch.tensor(weight_slice)
        self.input_slice_method = torch.tensor(input_slice)
        self.input_paral_size = input_paral_size
        self.input_quant_gran = input_quant_gran
        self.weight_sliced = SlicedData(self.weight_slice_method, device=device, bw_e=bw_e, is_weight=True,
                                        paral_size=weight_paral_size, quant_gran=weight_quant_gran)
        self.engine = engine
        self.weight_sliced.slice_data_imp(engine, self.weight.reshape(self.weight.shape[0], -1).detach().t())
        self.inference_mode = False

    def reset_parameters(self) -> None:
        torch.nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            fan_in, _ = torch.nn.init._calculate_fan_in_and_fan_out(self.weight)
            bound = 1 / math.sqrt(fan_in)
            torch.nn.init.uniform_(self.bias, -bound, bound)

    @property
    def _stride2(self):
        return _pair(self.stride)

    @property
    def _padding2(self):
        return _pair(self.padding)

    @property
    def _dilation2(self):
        return _pair(self.dilation)

    def _cim_forward(self, input, bias, inference=False):
        kh, kw = self.weight.shape[2], self.weight.shape[3]
        (sh, sw), (ph, pw), (dh, dw) = self._stride2, self._padding2, self._dilation2
        n, _, h, w = input.shape
        h_out = (h + 2 * ph - dh * (kh - 1) - 1) // sh + 1
        w_out = (w + 2 * pw - dw * (kw - 1) - 1) // sw + 1
        x_sliced = SlicedData(self.input_slice_method, device=input.device, bw_e=self.weight_sliced.bw_e,
                              is_weight=False, paral_size=self.input_paral_size, quant_gran=self.input_quant_gran,
                              inference=inference)
        # the input is sliced for exactly one multiply: with voltage noise on, the slicing applies that
        # multiply's noise (drawn with the seed the multiply would draw) and the separate pass is skipped
        noise_seed = int(torch.randint(0, 2 ** 62, (1,)).item()) if self.engine.conv_input_noise_fused() else None
        x_sliced._slice_conv_imp(self.engine, input.detach(), (kh, kw), (sh, sw), (ph, pw), (dh, dw),
                                 noise_seed=noise_seed)
        L = h_out * w_out
        cout = self.out_channels
        out = torch.empty((n, cout, h_out, w_out), dtype=torch.float32, device=self.engine.device)
        layout = N.OutLayout(L, cout * L, 1, L)
        b = None if bias is None else bias.detach().float()
        self.engine.MapReduceDot(x_sliced, self.weight_sliced, out=out, bias=b, layout=layout)
        return out, x_sliced

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        if self.inference_mode:
            return self._forward_inference(input)
        return conv2d_mem_func(self.engine, input, self.weight, self, self.bias)

    def _forward_inference(self, input: torch.Tensor) -> torch.Tensor:
        out, _ = self._cim_forward(input, self.bias, inference=True)
        return out

    def update_weight(self):
        self.weight_sliced.slice_data_imp(
            self.engine, self.weight.reshape(self.weight.shape[0], -1).detach().t().to(self.engine.device))
