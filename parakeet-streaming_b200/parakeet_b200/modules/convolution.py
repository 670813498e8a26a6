"""Conformer convolution module over the slot conv cache.

Drop-in for ``ConformerConvolution`` (parakeet/modules/convolution.py:107-162):
same submodule names (``pointwise_conv1``, ``depthwise_conv``, ``batch_norm``,
``pointwise_conv2``) and ``forward(x, pad_mask, cache) -> (x, cache)``.  The
two pointwise convs stay GEMMs; GLU, the pad mask, the cached causal
depthwise conv (CausalConv1d.update_cache, convolution.py:37-52), the
LayerNorm and the SiLU run as one libpk kernel that updates the conv cache
in place by slot.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from .cache import ConvCacheRef
from .feedforward import residual_linear


class ConformerConvolution(nn.Module):
    def __init__(self, hidden_size, kernel_size, use_bias=False):
        super().__init__()
        if use_bias:
            raise NotImplementedError("biased convs are not used by the streaming models")
        self.d_model = hidden_size
        self.kernel_size = kernel_size
        self.pointwise_conv1 = nn.Conv1d(hidden_size, 2 * hidden_size, 1, bias=False)
        self.depthwise_conv = nn.Conv1d(hidden_size, hidden_size, kernel_size, groups=hidden_size,
                                        bias=False)
        self.batch_norm = nn.LayerNorm(hidden_size)
        self.activation = nn.SiLU()
        self.pointwise_conv2 = nn.Conv1d(hidden_size, hidden_size, 1, bias=False)

    def forward(self, x: Tensor, pad_mask=None, cache: ConvCacheRef = None):
        if not isinstance(cache, ConvCacheRef):
            raise TypeError("ConformerConvolution needs the paged cache's conv handle")
        c = cache.cache
        h = F.linear(x, self.pointwise_conv1.weight[:, :, 0])            # [B, T, 2D]
        y = c.pool.conv_step(cache.layer_idx, h, self.depthwise_conv.weight, c.slots, c.lengths,
                             self.batch_norm.weight, self.batch_norm.bias, self.batch_norm.eps)
        return F.linear(y, self.pointwise_conv2.weight[:, :, 0]), cache

    def forward_residual(self, res: Tensor, x: Tensor, cache: ConvCacheRef = None) -> Tensor:
        """res + forward(x)[0] with the residual add in pointwise_conv2's GEMM
        (encoder.py:71-74)."""
        if not isinstance(cache, ConvCacheRef):
            raise TypeError("ConformerConvolution needs the paged cache's conv handle")
        c = cache.cache
        h = F.linear(x, self.pointwise_conv1.weight[:, :, 0])            # [B, T, 2D]
        y = c.pool.conv_step(cache.layer_idx, h, self.depthwise_conv.weight, c.slots, c.lengths,
                             self.batch_norm.weight, self.batch_norm.bias, self.batch_norm.eps)
        return residual_linear(res, y, None, weight=self.pointwise_conv2.weight[:, :, 0])


__all__ = ["ConformerConvolution"]
