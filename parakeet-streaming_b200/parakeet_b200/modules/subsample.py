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

from .._lib import check, lib
from ..ops import DTYPES, _stream


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

    def stream_supported(self, x: Tensor) -> bool:
        """The fused streaming path takes the 8x dw_striding stack with 3x3
        stride-2 convs and channels in multiples of 16, on CUDA."""
        return (x.is_cuda and x.dtype in DTYPES and self.sampling_num == 3
                and self._kernel_size == 3 and self._stride == 2
                and self._conv_channels % 16 == 0
                and self.conv[0].weight.dtype == x.dtype)

    def _out_weight(self) -> Tensor:
        """``out.weight`` with its columns reordered from (channel, frequency)
        to (frequency, channel), so channels-last rows multiply it directly;
        cached while the weight is unchanged."""
        w = self.out.weight
        try:
            version = w._version
        except RuntimeError:   # an inference-mode tensor has no version counter
            version = None
        key = (w.data_ptr(), version, w.dtype)
        if getattr(self, "_outw_key", None) != key:
            C = self._conv_channels
            f3 = w.shape[1] // C
            self._outw = w.reshape(w.shape[0], C, f3).transpose(1, 2).reshape(w.shape[0], -1).contiguous()
            self._outw_key = key
        return self._outw

    def forward_stream(self, xw: Tensor, drop: int = 0) -> Tensor:
        """``forward_full`` for a batch of streaming windows given as the
        pre-encode cache kernel writes them, xw [B, feat_in, frames], minus
        the first ``drop`` output frames: [B, frames' - drop, hidden].  conv1
        and the depthwise conv2 run as one libpk launch (conv1's activation
        stays in shared memory), the depthwise conv3 as another, the
        pointwise convs and ``out`` as GEMMs over channels-last rows; only the
        rows the kept outputs read are computed."""
        B, Fi, W = xw.shape
        C = self._conv_channels
        t1, f1 = W // 2 + 1, Fi // 2 + 1
        t2, f2 = t1 // 2 + 1, f1 // 2 + 1
        t3, f3 = t2 // 2 + 1, f2 // 2 + 1
        if not 0 <= drop < t3:
            raise ValueError(f"drop {drop} of {t3} output frames")
        first3 = drop
        first2 = max(0, 2 * first3 - 2)
        dt, dev, st = DTYPES[xw.dtype], xw.device, _stream(xw.device)
        c0, dw2, pw2, dw3, pw3 = self.conv[0], self.conv[2], self.conv[3], self.conv[5], self.conv[6]
        y2 = torch.empty(B, t2 - first2, f2, C, dtype=xw.dtype, device=dev)
        check(lib().pk_subsample_stage12(
            xw.data_ptr(), xw.stride(0), xw.stride(1), xw.stride(2), B, W, Fi,
            c0.weight.data_ptr(), c0.bias.data_ptr(), dw2.weight.data_ptr(), dw2.bias.data_ptr(),
            C, first2, y2.data_ptr(), dt, st), "pk_subsample_stage12")
        h2 = torch.addmm(pw2.bias, y2.view(-1, C), pw2.weight.view(C, C).t()).relu_()
        y3 = torch.empty(B, t3 - first3, f3, C, dtype=xw.dtype, device=dev)
        check(lib().pk_subsample_dw(
            h2.data_ptr(), B, t2, first2, f2, dw3.weight.data_ptr(), dw3.bias.data_ptr(), C,
            first3, y3.data_ptr(), dt, st), "pk_subsample_dw")
        h3 = torch.addmm(pw3.bias, y3.view(-1, C), pw3.weight.view(C, C).t()).relu_()
        out = torch.addmm(self.out.bias, h3.view(-1, f3 * C), self._out_weight().t())
        return out.view(B, t3 - first3, -1)


__all__ = ["ConvSubsampling"]
