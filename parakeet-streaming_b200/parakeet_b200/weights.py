"""Seeded random initialisation of the FastConformer encoder weights.

No checkpoint is reachable offline, so every run (tests, golden vectors,
benchmarks) uses synthetic weights.  Keys follow the reference's
``ConformerEncoder.state_dict()`` layout (``layers.{i}.<module>.<param>``,
see parakeet/modules/encoder.py:11-81 and parakeet/model.py:41-66 for the
fused ``self_attn.qkv.weight``), so one state_dict feeds both the reference
modules and this package.  numpy's PCG64 stream makes the values identical on
every machine for a given seed.
"""
from __future__ import annotations

import numpy as np


def _lin(rng, out_f, in_f):
    return (rng.standard_normal((out_f, in_f)) / np.sqrt(in_f)).astype(np.float32)


def _ln(rng, d):
    return ((1.0 + 0.05 * rng.standard_normal(d)).astype(np.float32),
            (0.05 * rng.standard_normal(d)).astype(np.float32))


def random_layer_state_dict(rng, dim, heads, ff_mult=4, conv_kernel=9):
    """One ConformerLayer's parameters (no biases: ``use_bias=False``,
    parakeet/config.py:17), float32 numpy arrays."""
    d_ff = dim * ff_mult
    dh = dim // heads
    sd = {}
    for name in ("norm_feed_forward1", "norm_self_att", "norm_conv",
                 "norm_feed_forward2", "norm_out"):
        sd[f"{name}.weight"], sd[f"{name}.bias"] = _ln(rng, dim)
    for ff in ("feed_forward1", "feed_forward2"):
        sd[f"{ff}.linear1.weight"] = _lin(rng, d_ff, dim)
        sd[f"{ff}.linear2.weight"] = _lin(rng, dim, d_ff)
    sd["self_attn.qkv.weight"] = _lin(rng, 3 * dim, dim)
    sd["self_attn.linear_pos.weight"] = _lin(rng, dim, dim)
    sd["self_attn.linear_out.weight"] = _lin(rng, dim, dim)
    sd["self_attn.pos_bias_u"] = (0.1 * rng.standard_normal((heads, dh))).astype(np.float32)
    sd["self_attn.pos_bias_v"] = (0.1 * rng.standard_normal((heads, dh))).astype(np.float32)
    sd["conv.pointwise_conv1.weight"] = _lin(rng, 2 * dim, dim)[:, :, None]
    sd["conv.depthwise_conv.weight"] = (rng.standard_normal((dim, 1, conv_kernel))
                                        / np.sqrt(conv_kernel)).astype(np.float32)
    sd["conv.batch_norm.weight"], sd["conv.batch_norm.bias"] = _ln(rng, dim)
    sd["conv.pointwise_conv2.weight"] = _lin(rng, dim, dim)[:, :, None]
    return sd


def random_encoder_layers(seed, num_layers, dim, heads, ff_mult=4, conv_kernel=9):
    """``{"layers.{i}.<key>": array}`` for ``num_layers`` layers."""
    rng = np.random.default_rng(seed)
    sd = {}
    for i in range(num_layers):
        for k, v in random_layer_state_dict(rng, dim, heads, ff_mult, conv_kernel).items():
            sd[f"layers.{i}.{k}"] = v
    return sd


def seeded_normal(seed, shape, scale=1.0, dtype=np.float32):
    """Synthetic activations: N(0, 1) * scale from a PCG64 stream."""
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(dtype)


def random_decoder_state_dict(seed, enc_dim, pred_dim=640, joint_dim=640, vocab_size=1026,
                              pred_layers=1, blank_bias=0.0):
    """Prediction network + joint network parameters with the keys of the
    reference's ``Predictor`` and ``Joiner`` state_dicts
    (parakeet/modules/decoder.py:5-86): an embedding of vocab_size + 1 rows
    (the blank row, the padding index, is zero), a ``pred_layers``-layer LSTM,
    and the joint's enc / pred projections and output layer over vocab_size + 1
    classes.  ``blank_bias`` is added to the blank class's output bias; random
    weights otherwise almost never emit blank."""
    rng = np.random.default_rng(seed)
    sd = {}
    emb = rng.standard_normal((vocab_size + 1, pred_dim)).astype(np.float32)
    emb[vocab_size] = 0.0
    sd["predictor.prediction.embed.weight"] = emb
    for k in range(pred_layers):
        sd[f"predictor.prediction.dec_rnn.weight_ih_l{k}"] = _lin(rng, 4 * pred_dim, pred_dim)
        sd[f"predictor.prediction.dec_rnn.weight_hh_l{k}"] = _lin(rng, 4 * pred_dim, pred_dim)
        sd[f"predictor.prediction.dec_rnn.bias_ih_l{k}"] = (
            0.1 * rng.standard_normal(4 * pred_dim)).astype(np.float32)
        sd[f"predictor.prediction.dec_rnn.bias_hh_l{k}"] = (
            0.1 * rng.standard_normal(4 * pred_dim)).astype(np.float32)
    sd["joiner.pred.weight"] = _lin(rng, joint_dim, pred_dim)
    sd["joiner.pred.bias"] = (0.1 * rng.standard_normal(joint_dim)).astype(np.float32)
    sd["joiner.enc.weight"] = _lin(rng, joint_dim, enc_dim)
    sd["joiner.enc.bias"] = (0.1 * rng.standard_normal(joint_dim)).astype(np.float32)
    sd["joiner.joint_net.2.weight"] = _lin(rng, vocab_size + 1, joint_dim)
    out_b = (0.1 * rng.standard_normal(vocab_size + 1)).astype(np.float32)
    out_b[vocab_size] += np.float32(blank_bias)
    sd["joiner.joint_net.2.bias"] = out_b
    return sd


def random_pre_encode_state_dict(seed, feat_in=128, channels=256, hidden=512, factor=8):
    """``ConvSubsampling`` parameters (parakeet/modules/subsample.py:61-150) with
    the reference's keys: conv.0 (1 -> channels, 3x3 stride 2), then per further
    factor of 2 a depthwise 3x3 stride-2 conv (conv.2, conv.5, ...) and a
    pointwise 1x1 conv (conv.3, conv.6, ...), and the output projection ``out``
    from channels x final frequency bins to ``hidden``."""
    rng = np.random.default_rng(seed)
    sd = {"conv.0.weight": (rng.standard_normal((channels, 1, 3, 3)) / 3.0).astype(np.float32),
          "conv.0.bias": (0.1 * rng.standard_normal(channels)).astype(np.float32)}
    idx, freq = 2, (feat_in + 2 + 1 - 3) // 2 + 1
    for _ in range(int(round(np.log2(factor))) - 1):
        sd[f"conv.{idx}.weight"] = (rng.standard_normal((channels, 1, 3, 3)) / 3.0).astype(np.float32)
        sd[f"conv.{idx}.bias"] = (0.1 * rng.standard_normal(channels)).astype(np.float32)
        sd[f"conv.{idx + 1}.weight"] = _lin(rng, channels, channels)[:, :, None, None]
        sd[f"conv.{idx + 1}.bias"] = (0.1 * rng.standard_normal(channels)).astype(np.float32)
        idx += 3
        freq = (freq + 2 + 1 - 3) // 2 + 1
    sd["out.weight"] = _lin(rng, hidden, channels * freq)
    sd["out.bias"] = (0.1 * rng.standard_normal(hidden)).astype(np.float32)
    return sd


def random_model_state_dict(seed, layers, dim, heads, vocab_size, pred_layers, feat_in=128,
                            sub_channels=256, pred_dim=640, joint_dim=640, blank_bias=0.0):
    """A whole ``Parakeet`` model's parameters (parakeet/model.py:69-102) with
    its state_dict keys: ``encoder.layers.*`` (seed), ``encoder.pre_encode.*``
    (seed + 1), ``predictor.*`` and ``joiner.*`` (seed + 2)."""
    sd = {f"encoder.{k}": v for k, v in random_encoder_layers(seed, layers, dim, heads).items()}
    sd.update({f"encoder.pre_encode.{k}": v for k, v in
               random_pre_encode_state_dict(seed + 1, feat_in, sub_channels, dim).items()})
    sd.update(random_decoder_state_dict(seed + 2, dim, pred_dim, joint_dim, vocab_size,
                                        pred_layers, blank_bias))
    return sd
