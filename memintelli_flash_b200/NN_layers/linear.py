"""``LinearMem``: CIM fully connected layer (memintelli/NN_layers/linear.py:18-85)."""
import math

import torch
import torch.nn as nn

from ..pimpy.data_formats import SlicedData
from .functions import linear_mem_func


class LinearMem(nn.Module):
    def __init__(self, engine, in_features: int, out_features: int, input_slice, weight_slice,
                 bias: bool = True, device=None, dtype=torch.float32, bw_e=None, input_paral_size=(1, 32),
                 weight_paral_size=(32, 32), input_quant_gran=(1, 32), weight_quant_gran=(32, 32)):
        super().__init__()
        factory_kwargs = {'device': device, 'dtype': dtype}
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.empty((out_features, in_features), **factory_kwargs))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, **factory_kwargs))
        else:
            self.register_parameter('bias', None)
        self.reset_parameters()
        self.weight_slice_method = torch.tensor(weight_slice)
        self.input_slice_method = torch.tensor(input_slice)
        self.weight_sliced = SlicedData(self.weight_slice_method, device=device, bw_e=bw_e, is_weight=True,
                                        paral_size=weight_paral_size, quant_gran=weight_quant_gran)
        self.engine = engine
        self.weight_sliced.slice_data_imp(engine, self.weight.detach().t())
        self.input_paral_size = input_paral_size
        self.input_quant_gran = input_quant_gran
        self.inference_mode = False

    def reset_parameters(self) -> None:
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            fan_in, _ = nn.init._calculate_fan_in_and_fan_out(self.weight)
            bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
            nn.init.uniform_(self.bias, -bound, bound)

    def _input_sliced(self, input, inference):
        return SlicedData(self.input_slice_method, device=input.device, bw_e=self.weight_sliced.bw_e,
                          is_weight=False, paral_size=self.input_paral_size, quant_gran=self.input_quant_gran,
                          inference=inference)

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        if self.inference_mode:
            return self._forward_inference(input)
        input_sliced = self._input_sliced(input, False)
        input_sliced.slice_data_imp(self.engine, input.detach())
        return linear_mem_func(self.engine, input, self.weight, input_sliced, self.weight_sliced, self.bias)

    def new_input(self):
        """An empty input SlicedData with this layer's input slicing, for the engine's fused
        producers (``DPETensor.slice_rmsnorm_input`` / ``slice_swiglu_input``)."""
        return SlicedData(self.input_slice_method, device=self.engine.device, bw_e=self.weight_sliced.bw_e,
                          is_weight=False, paral_size=self.input_paral_size, quant_gran=self.input_quant_gran,
                          inference=True)

    def forward_sliced(self, input_sliced) -> torch.Tensor:
        """Inference forward of an input already sliced (by ``new_input`` + a fused producer)."""
        bias = None if self.bias is None else self.bias.detach().float()
        return self.engine.MapReduceDot(input_sliced, self.weight_sliced, bias=bias)

    def _forward_inference(self, input: torch.Tensor) -> torch.Tensor:
        """Inference forward: the bias add is fused into the kernel's output store."""
        input_sliced = self._input_sliced(input, True)
        input_sliced.slice_data_imp(self.engine, input)
        bias = None if self.bias is None else self.bias.detach().float()
        return self.engine.MapReduceDot(input_sliced, self.weight_sliced, bias=bias)

    def update_weight(self):
        self.weight_sliced.slice_data_imp(self.engine, self.weight.detach().t().to(self.engine.device))
