"""float64 numpy restatement of the reference's streaming encoder hot path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Every function cites
the reference file and lines it restates; paths are relative to the
odunola499/parakeet-streaming source tree.

Shapes follow the reference: B streams in the batch, L layers, T frames in
the current chunk (= right context + 1), left context ``left`` (70),
window W = left + T, model width D, H heads of dh = D / H.
"""
from __future__ import annotations

import math
from collections import deque

import numpy as np

F64 = np.float64


# --------------------------------------------------------------------------
# Dense window cache  (parakeet/modules/cache.py:7-77)
# --------------------------------------------------------------------------
class DenseModelCache:
    """``ModelCache``: one dense K/V window and conv cache per slot.

    attn_k / attn_v: [slots, L, left + right + 1, D]   (cache.py:24-29)
    conv:            [slots, L, D, kernel - 1]         (cache.py:30-34)
    """

    def __init__(self, num_layers, att_context, dim, conv_kernel, slots=1,
                 dtype=F64):
        self.left = int(att_context[0])
        self.right = int(att_context[1])
        self.window = self.left + self.right + 1
        self.conv_len = int(conv_kernel - 1)
        self.attn_k = np.zeros((slots, num_layers, self.window, dim), dtype)
        self.attn_v = np.zeros_like(self.attn_k)
        self.conv = np.zeros((slots, num_layers, dim, self.conv_len), dtype)

    def update_attn_cache(self, layer, key, value):
        """cache.py:36-45: window[:left] <- window[-left:]; window[left:] <- new.

        ``key``/``value`` are [B, T, D] with T = right + 1 (a shorter chunk
        broadcasts along T exactly as ``Tensor.copy_`` does)."""
        left = self.left
        for buf, new in ((self.attn_k, key), (self.attn_v, value)):
            buf[:, layer, :left] = buf[:, layer, -left:].copy()
            buf[:, layer, left:] = new
        return self.attn_k[:, layer], self.attn_v[:, layer]

    def get_conv_cache(self, layer):            # cache.py:47-48
        return self.conv[:, layer]

    def update_conv_cache(self, layer, state):  # cache.py:50-53
        if state is not None:
            self.conv[:, layer] = state

    def reset_slot(self, slot):                 # cache.py:60-63
        self.attn_k[slot] = 0
        self.attn_v[slot] = 0
        self.conv[slot] = 0


class StreamingStateModel:
    """``StreamingState`` (cache.py:80-89) with the pool/batch tensors as numpy."""

    def __init__(self, cache, slots):
        self.cache = cache
        self.processed_frames = np.zeros(slots, np.int64)
        self.cache_lengths = np.zeros(slots, np.int64)


# --------------------------------------------------------------------------
# Slot scheduler  (parakeet/engine/scheduler.py:68-201)
# --------------------------------------------------------------------------
class SlotSchedulerModel:
    """FIFO slot free list, zero-on-acquire/release, gather/scatter by slot.

    init_state_pool: free = deque(range(pool))            scheduler.py:68-84
    acquire: popleft, then zero the slot                  scheduler.py:93-99
    release: zero the slot, then append                   scheduler.py:101-104
    pack:    index_select of every state tensor           scheduler.py:128-170
    unpack:  index_copy_ back                             scheduler.py:172-201
    """

    def __init__(self, num_layers, att_context, dim, conv_kernel, pool_size):
        self.pool = StreamingStateModel(
            DenseModelCache(num_layers, att_context, dim, conv_kernel, pool_size),
            pool_size)
        self.free = deque(range(pool_size))

    def _reset(self, slot):
        self.pool.processed_frames[slot] = 0
        self.pool.cache_lengths[slot] = 0
        self.pool.cache.reset_slot(slot)

    def acquire_state_slot(self):
        if not self.free:
            return None
        slot = self.free.popleft()
        self._reset(slot)
        return slot

    def release_state_slot(self, slot):
        self._reset(slot)
        self.free.append(slot)

    def pack_states(self, slots):
        idx = np.asarray(slots, np.int64)
        c = self.pool.cache
        batch = DenseModelCache(c.attn_k.shape[1], (c.left, c.right),
                                c.attn_k.shape[3], c.conv_len + 1, len(idx))
        batch.attn_k = c.attn_k[idx].copy()
        batch.attn_v = c.attn_v[idx].copy()
        batch.conv = c.conv[idx].copy()
        st = StreamingStateModel(batch, len(idx))
        st.processed_frames = self.pool.processed_frames[idx].copy()
        st.cache_lengths = self.pool.cache_lengths[idx].copy()
        return st, idx

    def unpack_states(self, st, idx):
        c = self.pool.cache
        self.pool.processed_frames[idx] = st.processed_frames
        self.pool.cache_lengths[idx] = st.cache_lengths
        c.attn_k[idx] = st.cache.attn_k
        c.attn_v[idx] = st.cache.attn_v
        c.conv[idx] = st.cache.conv


# --------------------------------------------------------------------------
# Streaming masks  (parakeet/modules/encoder.py:167-227)
# --------------------------------------------------------------------------
def streaming_masks(current_len, cache_lengths, processed_frames, lengths,
                    att_context):
    """Returns (pad_mask [B, T] bool, att_mask [B, T, left + T] bool); True
    means masked.  Same per-stream construction as encoder.py:186-225."""
    left, right = int(att_context[0]), int(att_context[1])
    chunk = right + 1
    left_chunks = left // chunk
    B = len(cache_lengths)
    kmax = left + current_len
    pad = np.zeros((B, current_len), bool)
    att = np.ones((B, current_len, kmax), bool)
    for b in range(B):
        c = int(cache_lengths[b])
        p = int(processed_frames[b])
        key_start = max(p - c, 0)
        key_len = c + current_len
        key_pos = np.arange(key_start, key_start + key_len)
        q_pos = key_pos[-current_len:]
        diff = (q_pos // chunk)[:, None] - (key_pos // chunk)[None, :]
        allowed = (diff <= left_chunks) & (diff >= 0)
        valid_cur = np.arange(current_len) < int(lengths[b])
        pad[b] = ~valid_cur
        valid_tot = np.zeros(key_len, bool)
        valid_tot[:c] = True
        valid_tot[c:] = valid_cur
        off = left - c
        allowed_full = np.zeros((current_len, kmax), bool)
        allowed_full[:, off:off + key_len] = allowed
        valid_full = np.zeros(kmax, bool)
        valid_full[off:off + key_len] = valid_tot
        allowed_full &= valid_cur[:, None] & valid_full[None, :]
        att[b] = ~allowed_full
    return pad, att


# --------------------------------------------------------------------------
# Relative positional encoding  (parakeet/modules/attention.py:23-62)
# --------------------------------------------------------------------------
def rel_pos_table(hidden, max_len, dtype=np.float32):
    """extend_pe + create_pe (attention.py:33-53): rows are relative
    positions max_len-1 ... -(max_len-1); even columns sin, odd cos.
    Computed in float32 like the reference's buffer."""
    positions = np.arange(max_len - 1, -max_len, -1, dtype=np.float32)[:, None]
    div = np.exp(np.arange(0, hidden, 2, dtype=np.float32)
                 * np.float32(-(math.log(10000.0) / hidden)))
    pe = np.zeros((positions.shape[0], hidden), np.float32)
    pe[:, 0::2] = np.sin(positions * div)
    pe[:, 1::2] = np.cos(positions * div)
    return pe.astype(dtype)


def pos_emb_slice(pe, cur_len, cache_len):
    """attention.py:55-62: the 2 * (cur_len + cache_len) - 1 rows centred on
    relative position 0; row p holds relative position (cur_len+cache_len-1) - p."""
    input_len = cur_len + cache_len
    center = pe.shape[0] // 2 + 1
    return pe[center - input_len:center + input_len - 1]


def rel_shift(x):
    """attention.py:79-83 (pad one column on the left, re-view, drop a row):
    out[..., i, j] = x[..., i, j + qlen - 1 - i]."""
    *lead, qlen, plen = x.shape
    xp = np.concatenate([np.zeros((*lead, qlen, 1), x.dtype), x], axis=-1)
    xp = xp.reshape(*lead, -1, qlen)[..., 1:, :]
    return xp.reshape(*lead, qlen, plen)


# --------------------------------------------------------------------------
# Rel-pos multi-head self-attention  (parakeet/modules/attention.py:9-125)
# --------------------------------------------------------------------------
def relpos_attention_core(q, k_win, v_win, pos_proj, bias_u, bias_v, att_mask,
                          num_heads, dtype=F64):
    """The part of ConformerAttention.forward between the qkv GEMM and
    linear_out (attention.py:99-122), in ``dtype`` (float64 as the checker;
    float32 when timed as the reference's CPU path).

    q: [B, T, D]; k_win, v_win: [B, W, D]; pos_proj = linear_pos(pos_emb):
    [P, D]; bias_u, bias_v: [H, dh]; att_mask [B, T, W] (True = masked).
    Returns [B, T, D] (heads concatenated, before linear_out)."""
    q = np.asarray(q, dtype)
    B, T, D = q.shape
    W = k_win.shape[1]
    H = num_heads
    dh = D // H
    qh = q.reshape(B, T, H, dh)
    kh = np.asarray(k_win, dtype).reshape(B, W, H, dh).transpose(0, 2, 1, 3)
    vh = np.asarray(v_win, dtype).reshape(B, W, H, dh).transpose(0, 2, 1, 3)
    P = pos_proj.shape[0]
    ph = np.asarray(pos_proj, dtype).reshape(1, P, H, dh).transpose(0, 2, 1, 3)
    qu = (qh + np.asarray(bias_u, dtype)).transpose(0, 2, 1, 3)  # [B,H,T,dh]
    qv = (qh + np.asarray(bias_v, dtype)).transpose(0, 2, 1, 3)
    bd = qv @ ph.transpose(0, 1, 3, 2)                           # [B,H,T,P]
    bd = rel_shift(bd)[..., :W] * (1.0 / math.sqrt(dh))
    mask = np.asarray(att_mask, bool)[:, None]                   # [B,1,T,W]
    bd = np.where(mask, -1e5, bd)
    # sdpa_attention_forward (attention.py:9-20): softmax(q k^T / sqrt(dh) + bias) v
    s = (qu @ kh.transpose(0, 1, 3, 2)) / math.sqrt(dh) + bd
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    o = p @ vh                                                   # [B,H,T,dh]
    return o.transpose(0, 2, 1, 3).reshape(B, T, D)


def relpos_attention(x, w, pos_emb, att_mask, cache, layer, num_heads):
    """ConformerAttention.forward (attention.py:85-125) with its weights in
    ``w`` (keys of ``self_attn.*``)."""
    x = np.asarray(x, F64)
    D = x.shape[-1]
    qkv = x @ np.asarray(w["qkv.weight"], F64).T                 # attention.py:94
    q, k, v = qkv[..., :D], qkv[..., D:2 * D], qkv[..., 2 * D:]
    k_win, v_win = cache.update_attn_cache(layer, k, v)          # attention.py:98
    pos_proj = np.asarray(pos_emb, F64) @ np.asarray(w["linear_pos.weight"], F64).T
    o = relpos_attention_core(q, k_win, v_win, pos_proj, w["pos_bias_u"],
                              w["pos_bias_v"], att_mask, num_heads)
    return o @ np.asarray(w["linear_out.weight"], F64).T         # attention.py:123


# --------------------------------------------------------------------------
# Convolution module  (parakeet/modules/convolution.py:8-52,107-162)
# --------------------------------------------------------------------------
def causal_depthwise_conv(x, cache, weight):
    """CausalConv1d.update_cache + forward (convolution.py:37-52) for the
    depthwise case (groups = D, no bias, right padding 0).

    x: [B, D, T]; cache: [B, D, K-1]; weight: [D, 1, K] -> (y [B, D, T],
    next_cache [B, D, K-1] = last K-1 columns of cat(cache, x))."""
    x = np.asarray(x, F64)
    cache = np.asarray(cache, F64)
    wk = np.asarray(weight, F64)[:, 0, :]                         # [D, K]
    K = wk.shape[1]
    full = np.concatenate([cache, x], axis=-1)                    # [B, D, K-1+T]
    T = x.shape[-1]
    y = np.zeros_like(x)
    for t in range(T):
        y[:, :, t] = (full[:, :, t:t + K] * wk[None]).sum(-1)
    return y, full[:, :, -cache.shape[-1]:].copy()


def layer_norm(x, weight, bias, eps=1e-5):
    x = np.asarray(x, F64)
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps) * np.asarray(weight, F64) + np.asarray(bias, F64)


def silu(x):
    return x / (1.0 + np.exp(-x))


def glu_channels(x):
    """F.glu(x, dim=1) on [B, 2D, T]: first half * sigmoid(second half)."""
    D = x.shape[1] // 2
    return x[:, :D] / (1.0 + np.exp(-x[:, D:]))


def conv_module(x, pad_mask, cache, w):
    """ConformerConvolution.forward (convolution.py:150-162); w holds the
    ``conv.*`` weights.  x: [B, T, D] -> ([B, T, D], next_cache)."""
    x = np.asarray(x, F64).transpose(0, 2, 1)                     # [B, D, T]
    pw1 = np.asarray(w["pointwise_conv1.weight"], F64)[:, :, 0]   # [2D, D]
    x = np.einsum("od,bdt->bot", pw1, x)
    x = glu_channels(x)
    x = np.where(np.asarray(pad_mask, bool)[:, None, :], 0.0, x)
    x, nxt = causal_depthwise_conv(x, cache, w["depthwise_conv.weight"])
    x = layer_norm(x.transpose(0, 2, 1), w["batch_norm.weight"],
                   w["batch_norm.bias"]).transpose(0, 2, 1)
    x = silu(x)
    pw2 = np.asarray(w["pointwise_conv2.weight"], F64)[:, :, 0]
    x = np.einsum("od,bdt->bot", pw2, x)
    return x.transpose(0, 2, 1), nxt


def feed_forward(x, w, prefix):
    """ConformerFeedForward.forward (feedforward.py:21-26), no biases."""
    h = np.asarray(x, F64) @ np.asarray(w[prefix + "linear1.weight"], F64).T
    return silu(h) @ np.asarray(w[prefix + "linear2.weight"], F64).T


# --------------------------------------------------------------------------
# Conformer layer and streaming encoder step  (parakeet/modules/encoder.py)
# --------------------------------------------------------------------------
def conformer_layer(x, w, layer, pos_emb, pad_mask, att_mask, cache, num_heads):
    """ConformerLayer.forward (encoder.py:50-81); ``w`` maps the layer's
    state_dict keys (without the ``layers.{i}.`` prefix) to arrays."""
    def ln(name, v):
        return layer_norm(v, w[name + ".weight"], w[name + ".bias"])

    res = np.asarray(x, F64).copy()
    res = res + 0.5 * feed_forward(ln("norm_feed_forward1", res), w, "feed_forward1.")
    att_w = {k[len("self_attn."):]: v for k, v in w.items() if k.startswith("self_attn.")}
    res = res + relpos_attention(ln("norm_self_att", res), att_w, pos_emb, att_mask,
                                 cache, layer, num_heads)
    conv_w = {k[len("conv."):]: v for k, v in w.items() if k.startswith("conv.")}
    y, nxt = conv_module(ln("norm_conv", res), pad_mask, cache.get_conv_cache(layer), conv_w)
    cache.update_conv_cache(layer, nxt)
    res = res + y
    res = res + 0.5 * feed_forward(ln("norm_feed_forward2", res), w, "feed_forward2.")
    return ln("norm_out", res)


def encoder_step(x, state, length, layer_weights, pe, att_context, num_heads):
    """ConformerEncoder.forward (encoder.py:229-267) for an already
    subsampled chunk x: [B, T, D]; ``state`` is a StreamingStateModel whose
    cache is a DenseModelCache.  Returns [B, D, T] and updates ``state``."""
    x = np.asarray(x, F64)
    T = x.shape[1]
    left = int(att_context[0])
    pos_emb = pos_emb_slice(pe, T, left)                         # encoder.py:239
    pad, att = streaming_masks(T, state.cache_lengths, state.processed_frames,
                               length, att_context)
    for i, w in enumerate(layer_weights):
        x = conformer_layer(x, w, i, pos_emb, pad, att, state.cache, num_heads)
    length = np.asarray(length, np.int64)
    state.processed_frames = state.processed_frames + length     # encoder.py:257-260
    state.cache_lengths = np.minimum(state.cache_lengths + length, left)
    return x.transpose(0, 2, 1)


def layer_weights_from_state_dict(sd, num_layers):
    """Split an encoder state_dict (``layers.{i}.*`` keys) per layer."""
    out = []
    for i in range(num_layers):
        p = f"layers.{i}."
        out.append({k[len(p):]: np.asarray(v) for k, v in sd.items() if k.startswith(p)})
    return out
