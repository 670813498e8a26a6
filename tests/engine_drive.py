"""Drives the reference engine's ``ModelRunner`` (parakeet/engine/model_runner.py)
synchronously over one stream of audio, as configs[0] specifies: pcm16 audio
pushed in 160 ms pieces through ``Sequence.push_samples`` and ``step()`` called
until the stream is idle after every push.  Used by the end-to-end golden
generator (the reference alone, CPU fp32) and by the GPU drop-in test (the same
``ModelRunner`` over this package's scheduler, encoder, features and decode),
so both sides see exactly the same call sequence.

Only observation is added: ``_decode_batch`` (model_runner.py:347) is wrapped
to record, per encoder chunk of the stream, the chunk it was given (the
encoder's output, ``[1, D, frames]``) and the token ids it returned."""
from __future__ import annotations

import numpy as np

SAMPLE_RATE = 16000


def pcm16_noise(seed: int, seconds: float, amplitude: int = 8000) -> np.ndarray:
    """White noise as pcm16 samples uniform in [-amplitude, amplitude], seeded
    PCG64, converted to float32 the way the reference server does
    (int16 / 32768, parakeet/server.py:442)."""
    n = int(round(seconds * SAMPLE_RATE))
    x = np.random.default_rng(seed).integers(-amplitude, amplitude + 1, n).astype(np.int16)
    return x.astype(np.float32) / np.float32(32768.0)


def drive(runner, audio: np.ndarray, push: int = 2560, max_steps: int = 100000):
    """Returns [(encoder chunk float32 [D, frames], token ids)] per encoder
    chunk of the stream, in decode order."""
    seq = runner.create_sequence()
    if seq is None:
        raise RuntimeError("no free stream slot")
    runner.add_sequence(seq)
    record = []
    inner = runner._decode_batch

    def recording(seqs, chunks):
        lists = inner(seqs, chunks)
        for s, c, toks in zip(seqs, chunks, lists):
            if s is seq:
                record.append((c.detach().float().cpu().numpy()[0], [int(t) for t in toks]))
        return lists

    runner._decode_batch = recording
    steps = 0
    try:
        for start in range(0, len(audio), push):
            piece = audio[start:start + push]
            with seq.lock:
                seq.push_samples(piece, final=start + push >= len(audio))
            while seq.raw_queue or seq.has_chunk_ready() or seq.encoded_queue:
                runner.step()
                steps += 1
                if steps > max_steps:
                    raise RuntimeError("stream did not go idle")
    finally:
        runner._decode_batch = inner
    return record


def pack(record):
    """Flattens a ``drive`` record into arrays: tokens, per-chunk offsets into
    them, per-chunk frame counts and the encoder outputs [D, sum(frames)]."""
    toks, offsets, frames, enc = [], [0], [], []
    for chunk, t in record:
        toks.extend(t)
        offsets.append(len(toks))
        frames.append(chunk.shape[1])
        enc.append(chunk)
    return {"tokens": np.array(toks, np.int64), "offsets": np.array(offsets, np.int64),
            "frames": np.array(frames, np.int64),
            "enc": np.concatenate(enc, axis=1).astype(np.float32)}
