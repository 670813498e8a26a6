"""Convolutional subsampling (the pre-encoder): drop-in for ``ConvSubsampling``
(parakeet/modules/subsample.py:61-179) with the same constructor arguments and
parameter names (``conv.{0,2,3,5,6,...}``, ``out``), so reference state_dicts
load unchanged.

Every conv is causal in time and frequency as ``CausalConv2D``
(parakeet/modules/convolution.py:55-104): zero padding of kernel-1 before and
stride-1 after the input on both axes.  Frames at or beyond a row's length are
zeroed before every layer and at the end (``MaskedConvSequential``,
subsample.py:32-58), with the lengths advanced through every strided layer."""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor, nn


class ConvSubsampling(nn.Module):
    def __init__(self, hidden_size: int, subsampling_conv_channels: int, feat_in: int,
                 subsampling_factor: int, stride: int = 2, kernel_size: int = 3):
        super().__init__()
        self.feat_in, self._conv_channels = feat_in, subsampling_conv_channels
        self.subsampling_factor = subsampling_factor
        self.sampling_num = int(math.log(subsampling_factor, 2))
        self._stride, self._kernel_size = stride, kernel_size
        self._left_padding, self._right_padding = kernel_size - 1, stride - 1
        ch = subsampling_conv_channels
        layers = [nn.Conv2d(1, ch, kernel_size, stride), nn.ReLU(inplace=True)]
        for _ in range(self.sampling_num - 1):
            layers += [nn.Conv2d(ch, ch, kernel_size, stride, groups=ch),   # depthwise
                       nn.Conv2d(ch, ch, 1, 1),                            # pointwise
                       nn.ReLU(inplace=True)]
        self.conv = nn.Sequential(*layers)
        freq = feat_in
        for _ in range(self.sampling_num):
            freq = self._out_len(freq)
        self.out = nn.Linear(ch * freq, hidden_size, bias=True)

    def _out_len(self, n: int) -> int:
        return (n + self._left_padding + self._right_padding - self._kernel_size) // self._stride + 1

    def forward(self, x: Tensor, lengths: Tensor):
        """x [B, frames, feat_in], lengths [B] -> ([B, frames', hidden], lengths')."""
        x = x.unsqueeze(1)                                   # [B, 1, time, freq]
        lengths = lengths.to(torch.long)
        pad = (self._left_padding, self._right_padding) * 2
        for layer in self.conv:
            if isinstance(layer, nn.Conv2d):
                x = x * (torch.arange(x.shape[2], device=x.device)[None, :] < lengths[:, None]
                         ).to(x.dtype)[:, None, :, None]
                if layer.kernel_size[0] > 1:
                    x = F.pad(x, pad)
                x = layer(x)
                if layer.stride[0] > 1:
                    lengths = (lengths + self._left_padding + self._right_padding
                               - self._kernel_size) // self._stride + 1
            else:
                x = layer(x)
        x = x * (torch.arange(x.shape[2], device=x.device)[None, :] < lengths[:, None]
                 ).to(x.dtype)[:, None, :, None]
        b, c, t, f = x.shape
        return self.out(x.transpose(1, 2).reshape(b, t, c * f)), lengths

    def forward_full(self, x: Tensor) -> Tensor:
        """``forward`` for a batch whose rows all span every frame (the
        streaming pre-encode: no masks to apply).  Channels-last activations;
        the causal padding is the conv's own symmetric padding of kernel-1 with
        the trailing output frame dropped when the causal length is shorter,
        which selects the same input windows as padding kernel-1 before and
        stride-1 after."""
        x = x.unsqueeze(1).contiguous(memory_format=torch.channels_last)
        for layer in self.conv:
            if isinstance(layer, nn.Conv2d) and layer.kernel_size[0] > 1:
                t, f = self._out_len(x.shape[2]), self._out_len(x.shape[3])
                x = F.conv2d(x, layer.weight, layer.bias, layer.stride, self._left_padding,
                             1, layer.groups)[:, :, :t, :f]
            else:
                x = layer(x)
        b, c, t, f = x.shape
        return self.out(x.permute(0, 2, 1, 3).reshape(b, t, c * f))


__all__ = ["ConvSubsampling"]
