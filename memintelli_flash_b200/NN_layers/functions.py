"""Autograd wrappers of the CIM layers (memintelli/NN_layers/functions.py:34-118, 97-343).

Forward runs the fused CIM kernels; backward is the reference's straight-through
estimator: plain GEMMs / convolutions on the dequantised operands.
"""
import torch
import torch.nn.functional as F


class LinearMemRunc(torch.autograd.Function):
    @staticmethod
    def forward(ctx, engine, input, weight, input_slice, weight_slice, bias):
        ctx.save_for_backward(input_slice.quantized_data, weight_slice.quantized_data, bias)
        return engine.MapReduceDot(input_slice, weight_slice, bias=None if bias is None else bias.detach().float())

    @staticmethod
    def backward(ctx, grad_output):
        input_quant, weight_quant, bias = ctx.saved_tensors
        grad_input = grad_weight = grad_bias = None
        if ctx.needs_input_grad[1]:
            grad_input = grad_output.matmul(weight_quant.T.to(grad_output.dtype))
        if ctx.needs_input_grad[2]:
            g2 = grad_output.reshape(-1, grad_output.shape[-1])
            grad_weight = g2.T.matmul(input_quant.reshape(-1, input_quant.shape[-1]).to(g2.dtype))
        if bias is not None and ctx.needs_input_grad[5]:
            grad_bias = grad_output.reshape(-1, grad_output.shape[-1]).sum(0)
        return None, grad_input, grad_weight, None, None, grad_bias


def linear_mem_func(engine, input, weight, input_slice, weight_slice, bias=None):
    return LinearMemRunc.apply(engine, input, weight, input_slice, weight_slice, bias)


class Conv2dMemRunc(torch.autograd.Function):
    @staticmethod
    def forward(ctx, engine, input, weight, layer, bias):
        out, x_sliced = layer._cim_forward(input, bias)
        wq = layer.weight_sliced.quantized_data                 # (C*kh*kw, Cout)
        xq = x_sliced.quantized_data                            # (N, L, C*kh*kw)
        ctx.save_for_backward(xq, wq, bias)
        ctx.geom = (input.shape, weight.shape, layer._stride2, layer._padding2, layer._dilation2)
        return out

    @staticmethod
    def backward(ctx, grad_output):
        xq, wq, bias = ctx.saved_tensors
        in_shape, w_shape, stride, padding, dilation = ctx.geom
        g = grad_output.reshape(grad_output.shape[0], grad_output.shape[1], -1)    # (N, Cout, L)
        grad_input = grad_weight = grad_bias = None
        if ctx.needs_input_grad[1]:
            cols = torch.matmul(wq.to(g.dtype), g)                                    # (N, C*kh*kw, L)
            grad_input = F.fold(cols, in_shape[2:], w_shape[2:], dilation=dilation, padding=padding, stride=stride)
        if ctx.needs_input_grad[2]:
            gw = torch.einsum("ncl,nlk->ck", g, xq.to(g.dtype))
            grad_weight = gw.reshape(w_shape)
        if bias is not None and ctx.needs_input_grad[4]:
            grad_bias = grad_output.sum((0, 2, 3))
        return None, grad_input, grad_weight, None, grad_bias


def conv2d_mem_func(engine, input, weight, layer, bias=None):
    return Conv2dMemRunc.apply(engine, input, weight, layer, bias)
