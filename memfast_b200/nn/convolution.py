"""Conv2d inference as an implicit GEMM on the programmed analog matrices.

The reference (memfast/nn/convolution.py:10-62) programs one matrix per channel
group, materialises ``F.unfold`` patches, multiplies each group's slice and
folds the result back.  Here the patch matrix never exists: each group's
patches are quantised straight from the NCHW input by ``mf_quantize_conv_input``
(same codes and scales as quantising the unfolded patches), the group's product
runs on those codes, and the output is returned as the same [B, O, OH, OW] view
of a [B*OH*OW, O] buffer that the reference's transpose/reshape gives.  Module
state (``matrices.<g>.*`` buffers and names ``<name>.group<g>``) matches the
reference, so checkpoints move between the two.
"""

import torch
from torch import nn
from torch.nn import functional as F

from .. import _lib
from ..quantization import conv_input_tiles


class AnalogConv2d(nn.Module):
    """Conv2d lowered to independently programmed matrices for each group."""

    def __init__(self, source, simulator, *, name="conv"):
        super().__init__()
        if not isinstance(source, nn.Conv2d):
            raise TypeError("source must be torch.nn.Conv2d")
        if isinstance(source.padding, str):
            raise ValueError("use numeric Conv2d padding before conversion")
        self.in_channels, self.out_channels = source.in_channels, source.out_channels
        self.kernel_size, self.stride = source.kernel_size, source.stride
        self.padding, self.dilation = source.padding, source.dilation
        self.groups, self.padding_mode = source.groups, source.padding_mode
        rows = source.out_channels // source.groups
        weight = source.weight.detach()
        bias = None if source.bias is None else source.bias.detach()
        self.matrices = nn.ModuleList(
            simulator.map(weight[g * rows:(g + 1) * rows].flatten(1),
                          bias=None if bias is None else bias[g * rows:(g + 1) * rows],
                          name=f"{name}.group{g}")
            for g in range(source.groups)
        )

    def _geometry(self, group, zero_padding):
        g = _lib.MFConv2d()
        g.kernel_h, g.kernel_w = self.kernel_size
        g.stride_y, g.stride_x = self.stride
        g.pad_h, g.pad_w = zero_padding
        g.dilation_h, g.dilation_w = self.dilation
        g.group_channels = self.in_channels // self.groups
        g.channel_begin = group * g.group_channels
        return g

    def _output_extent(self, height, width):
        extents = []
        for size, pad, dilation, kernel, stride in zip((height, width), self.padding, self.dilation,
                                                       self.kernel_size, self.stride):
            extents.append((size + 2 * pad - dilation * (kernel - 1) - 1) // stride + 1)
        return extents

    @torch.no_grad()
    def forward(self, x):
        if x.ndim != 4 or x.shape[1] != self.in_channels:
            raise ValueError("expected NCHW input with matching channels")
        if not x.is_floating_point():
            raise ValueError("input must be floating with matching in_features")
        first = self.matrices[0]
        if x.device != first.packed.device or x.device != first.simulator.device:
            raise ValueError("input and simulator must use the same device")
        batch = x.shape[0]
        out_h, out_w = self._output_extent(*x.shape[-2:])
        if out_h < 1 or out_w < 1:
            raise RuntimeError("convolution window larger than the padded input")
        if x.numel() == 0:
            return x.new_empty((batch, self.out_channels, out_h, out_w))
        zero_padding = self.padding
        if self.padding_mode != "zeros":
            pad_h, pad_w = self.padding
            x = F.pad(x, (pad_w, pad_w, pad_h, pad_h), mode=self.padding_mode)
            zero_padding = (0, 0)
        positions = out_h * out_w
        # The reference's tuned-mode key is the shape of the patches it multiplies.
        shape = (batch, positions, self.in_channels // self.groups * self.kernel_size[0] * self.kernel_size[1])
        parts = []
        for group, matrix in enumerate(self.matrices):
            codes, xscale, flag = conv_input_tiles(x, matrix.config, self._geometry(group, zero_padding),
                                                   matrix.input_scale)
            parts.append(matrix._product(codes, xscale, shape, x.dtype, input_flag=flag))
        rows = parts[0] if len(parts) == 1 else torch.cat(parts, dim=1)
        # [B*L, O] rows -> the [B, O, OH, OW] view (no copy), as transpose(1, 2).reshape does.
        return rows.view(batch, positions, self.out_channels).transpose(1, 2).reshape(
            batch, self.out_channels, out_h, out_w)
