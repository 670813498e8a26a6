"""Streaming FastConformer encoder over the paged cache.

Drop-in for ``ConformerLayer`` and ``ConformerEncoder``
(parakeet/modules/encoder.py:11-267): same constructor arguments, submodule
names and ``init_streaming_state`` / ``forward(x, state, length)``.

What changes on the path:
* no dense masks: ``_create_streaming_masks`` (encoder.py:167-227, a Python
  loop with two device syncs per stream) is gone; the attention kernel
  evaluates the same mask per (query, key) from the slot counters and the
  conv kernel applies the pad mask from ``length``;
* the cache is paged: one step starts with the page allocator kernel and
  ends with the counter update of encoder.py:257-260 on the device.
"""
from __future__ import annotations

import torch
from torch import Tensor, nn

from ..ops import PagedKVPool, layer_norm
from .attention import ConformerAttention, PositionalEncoding
from .cache import PagedModelCache, StreamingState
from .convolution import ConformerConvolution
from .feedforward import ConformerFeedForward
from .subsample import ConvSubsampling


class ConformerLayer(nn.Module):
    """FF/2 -> MHSA -> conv -> FF/2 -> LayerNorm (encoder.py:50-81)."""

    def __init__(self, layer_idx, hidden_size, d_ff, num_heads, dropout, conv_kernel_size, use_bias):
        super().__init__()
        self.layer_idx = layer_idx
        self.hidden_size = hidden_size
        self.norm_feed_forward1 = nn.LayerNorm(hidden_size)
        self.feed_forward1 = ConformerFeedForward(hidden_size, d_ff, dropout, use_bias)
        self.norm_conv = nn.LayerNorm(hidden_size)
        self.conv = ConformerConvolution(hidden_size, conv_kernel_size)
        self.norm_self_att = nn.LayerNorm(hidden_size)
        self.self_attn = ConformerAttention(layer_idx, num_heads, hidden_size, use_bias)
        self.norm_feed_forward2 = nn.LayerNorm(hidden_size)
        self.feed_forward2 = ConformerFeedForward(hidden_size, d_ff, dropout, use_bias)
        self.norm_out = nn.LayerNorm(hidden_size)

    def forward(self, x: Tensor, pos_emb: Tensor, pad_mask, attn_mask, cache: PagedModelCache):
        return self.forward_fused(x, layer_norm(x, self.norm_feed_forward1), pos_emb, cache)

    def forward_fused(self, x: Tensor, h: Tensor, pos_emb: Tensor, cache: PagedModelCache,
                      next_norm: nn.LayerNorm | None = None):
        """``forward`` given h = norm_feed_forward1(x).  The residual adds and
        the FF halves ride in the epilogue of each module's last GEMM
        (res + alpha * acc); the LayerNorms are libpk launches, and with
        ``next_norm`` (the next layer's norm_feed_forward1) the last one also
        returns that layer's h: (out, h_next)."""
        res = self.feed_forward1.forward_residual(x, h, 0.5)
        res = self.self_attn.forward_residual(res, layer_norm(res, self.norm_self_att), pos_emb,
                                              cache)
        conv_cache = cache.get_conv_cache(self.layer_idx)          # updated in place
        res = self.conv.forward_residual(res, layer_norm(res, self.norm_conv), conv_cache)
        res = self.feed_forward2.forward_residual(res, layer_norm(res, self.norm_feed_forward2), 0.5)
        return layer_norm(res, self.norm_out, next_norm)


class ConformerEncoder(nn.Module):
    def __init__(self, feat_in: int, hidden_size, ff_expansion_factor: int, num_layers: int,
                 num_heads: int, subsampling_factor: int, pos_emb_max_len: int,
                 conv_kernel_size: int, att_context_size, subsampling_conv_channels: int,
                 use_bias: bool, pre_encode_cache_size=(0, 9), drop_extra_pre_encoded: int = 2):
        super().__init__()
        self.embed_dim = hidden_size
        self.pre_encode = ConvSubsampling(hidden_size, subsampling_conv_channels, feat_in,
                                          subsampling_factor, stride=2, kernel_size=3)
        self.num_heads = num_heads
        self.feat_in = feat_in
        self.subsampling_factor = subsampling_factor
        self.subsampling_conv_channels = subsampling_conv_channels
        self.pos_enc = PositionalEncoding(hidden_size, 0.0, pos_emb_max_len, 0.0)
        self.pos_enc.extend_pe(pos_emb_max_len, device="cpu")
        d_ff = hidden_size * ff_expansion_factor
        self.layers = nn.ModuleList(
            ConformerLayer(i, hidden_size, d_ff, num_heads, 0.0, conv_kernel_size, use_bias)
            for i in range(num_layers))
        self.att_context_size = tuple(att_context_size)
        self.conv_kernel_size = conv_kernel_size
        self.pre_encode_cache_size = pre_encode_cache_size
        self.drop_extra_pre_encoded = drop_extra_pre_encoded

    @property
    def chunk_size(self) -> int:
        return self.att_context_size[1] + 1

    def make_pool(self, num_slots: int, device=None, dtype=None, **kw) -> PagedKVPool:
        p = next(self.parameters())
        return PagedKVPool(len(self.layers), self.embed_dim, self.num_heads, self.att_context_size,
                           num_slots, conv_kernel=self.conv_kernel_size,
                           dtype=dtype or p.dtype, device=device or p.device, **kw)

    def init_streaming_state(self, batch_size: int = 1, device=None, dtype=None, **pool_kw):
        """A fresh pool of ``batch_size`` slots and the state over all of them
        (encoder.py:140-165)."""
        pool = self.make_pool(batch_size, device, dtype, **pool_kw)
        slots = torch.arange(batch_size, dtype=torch.int32, device=pool.device)
        return StreamingState(PagedModelCache(pool, slots))

    def forward(self, x: Tensor, state: StreamingState, length: Tensor | None = None,
                bypass_pre_encode: bool = False):
        """x [B, T, D]: one chunk of subsampled frames per slot of ``state``.
        As in the reference (encoder.py:229-267), ``pre_encode`` is never run
        here whatever ``bypass_pre_encode`` says: the engine runs it per
        window (model_runner.py:221) and hands the encoder its frames."""
        cache = state.cache
        pool = cache.pool
        B, T = x.shape[:2]
        if T != pool.chunk:
            raise ValueError(f"chunk of {T} frames; this model steps {pool.chunk} at a time")
        if B != cache.batch_size:
            raise ValueError(f"batch {B} != {cache.batch_size} slots in the state")
        if length is None:
            length = torch.full((B,), T, dtype=torch.int32, device=pool.device)
        cache.lengths = torch.as_tensor(length).to(device=pool.device, dtype=torch.int32)
        pool.begin_step(cache.slots, cache.lengths)
        x, pos_emb = self.pos_enc(x, cache_len=self.att_context_size[0])
        h = layer_norm(x, self.layers[0].norm_feed_forward1)
        for i, layer in enumerate(self.layers):
            nxt = self.layers[i + 1].norm_feed_forward1 if i + 1 < len(self.layers) else None
            out = layer.forward_fused(x, h, pos_emb, cache, nxt)
            x, h = out if nxt is not None else (out, None)
        pool.end_step(cache.slots, cache.lengths)             # encoder.py:257-260
        return x.transpose(1, 2), state


__all__ = ["ConformerEncoder", "ConformerLayer"]
