"""The reference's CPU path for one isolated paged-attention step, timed as
the CPU baseline.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): imported by
``bench.py`` for its ``cpu_baseline`` leg and its ``--impl reference`` arm,
never by the product.

One step over B streams and L layers follows the reference's order:
``Scheduler.pack_states`` (index_select of the whole slot state,
parakeet/engine/scheduler.py:128-170), the streaming masks
(parakeet/modules/encoder.py:167-227), per layer the shift-append of
``ModelCache.update_attn_cache`` (parakeet/modules/cache.py:36-45) and the
rel-pos attention core (parakeet/modules/attention.py:99-122), the counter
update (encoder.py:257-260) and ``unpack_states`` (index_copy_ back,
scheduler.py:172-201).  float32, like the reference's CPU model.
"""
from __future__ import annotations

import numpy as np

from .streaming import SlotSchedulerModel, relpos_attention_core, streaming_masks


class ReferenceStep:
    def __init__(self, num_layers, dim, heads, att_context, num_streams, seed=1):
        self.L, self.D, self.H = num_layers, dim, heads
        self.att = att_context
        self.left, self.T = att_context[0], att_context[1] + 1
        self.B = num_streams
        self.sched = SlotSchedulerModel(num_layers, att_context, dim, 9, num_streams)
        c = self.sched.pool.cache
        c.attn_k = c.attn_k.astype(np.float32)
        c.attn_v = c.attn_v.astype(np.float32)
        c.conv = c.conv.astype(np.float32)
        self.slots = [self.sched.acquire_state_slot() for _ in range(num_streams)]
        rng = np.random.default_rng(seed)
        P = 2 * (self.left + self.T) - 1
        s = 1.0 / np.sqrt(dim // heads)
        self.pos = (rng.standard_normal((num_layers, P, dim)) * s).astype(np.float32)
        self.bu = (rng.standard_normal((num_layers, heads, dim // heads)) * s).astype(np.float32)
        self.bv = (rng.standard_normal((num_layers, heads, dim // heads)) * s).astype(np.float32)
        self.rng = rng

    def inputs(self):
        s = 1.0 / np.sqrt(self.D // self.H)
        return (self.rng.standard_normal((self.L, self.B, self.T, 3 * self.D)) * s).astype(np.float32)

    def step(self, qkv, lengths=None):
        """qkv: [L, B, T, 3D] float32 -> attention output [L, B, T, D]."""
        D = self.D
        lengths = np.full(self.B, self.T) if lengths is None else np.asarray(lengths)
        st, idx = self.sched.pack_states(self.slots)
        _, mask = streaming_masks(self.T, st.cache_lengths, st.processed_frames, lengths, self.att)
        out = np.empty((self.L, self.B, self.T, D), np.float32)
        for l in range(self.L):
            q, k, v = qkv[l, ..., :D], qkv[l, ..., D:2 * D], qkv[l, ..., 2 * D:]
            kw, vw = st.cache.update_attn_cache(l, k, v)
            out[l] = relpos_attention_core(q, kw, vw, self.pos[l], self.bu[l], self.bv[l], mask,
                                           self.H, dtype=np.float32)
        st.processed_frames = st.processed_frames + lengths
        st.cache_lengths = np.minimum(st.cache_lengths + lengths, self.left)
        self.sched.unpack_states(st, idx)
        return out
