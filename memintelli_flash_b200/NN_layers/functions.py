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
        """Straight-through gradients of Conv2dMemRunc.backward (functions.py:141-266).

        grad_input: transposed convolution of grad_output with the quantised weight.
        grad_weight: the reference first folds the quantised input patches back to an
        image, averaging the overlapping copies of each pixel (functions.py:151-160),
        then takes the convolution weight gradient against that image.
        """
        xq, wq, bias = ctx.saved_tensors
        in_shape, w_shape, stride, padding, dilation = ctx.geom
        g = grad_output.reshape(grad_output.shape[0], grad_output.shape[1], -1)    # (N, Cout, L)
        grad_input = grad_weight = grad_bias = None
        if ctx.needs_input_grad[1]:
            cols = torch.matmul(wq.to(g.dtype), g)                                    # (N, C*kh*kw, L)
            grad_input = F.fold(cols, in_shape[2:], w_shape[2:], dilation=dilation, padding=padding, stride=stride)
        if ctx.needs_input_grad[2]:
            fold = dict(kernel_size=tuple(w_shape[2:]), dilation=dilation, padding=padding, stride=stride)
            ones = torch.ones(in_shape, device=g.device, dtype=g.dtype)
            count = F.fold(F.unfold(ones, **fold), tuple(in_shape[2:]), **fold)
            count = torch.where(count == 0, torch.ones_like(count), count)
            image = F.fold(xq.transpose(1, 2).to(g.dtype), tuple(in_shape[2:]), **fold) / count
            grad_weight = torch.nn.grad.conv2d_weight(image, tuple(w_shape), grad_output, stride=stride,
                                                      padding=padding, dilation=dilation)
        if bias is not None and ctx.needs_input_grad[4]:
            grad_bias = grad_output.sum((0, 2, 3))
        return None, grad_input, grad_weight, None, grad_bias


def conv2d_mem_func(engine, input, weight, layer, bias=None):
    return Conv2dMemRunc.apply(engine, input, weight, layer, bias)
