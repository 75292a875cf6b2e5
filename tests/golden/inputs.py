"""Seeded synthetic inputs shared by the fixture generator and the tests.

There is no audio or real checkpoint here: log-mel frames are N(0, 1) of shape
[n_mels, 100*s + 1] for an utterance of s seconds, encoder outputs are N(0, 1),
and per-sequence output lengths are forced (EOS written at the drawn length).
"""
import importlib

import numpy as np

ctb = importlib.import_module("cohere-transcribe_b200")


def lcg_stream(seed: int = 0xDEADBEEF):
    """The reference kernel test's generator (tests/test_kernels.c:28-37):
    32-bit LCG, value = (float)(int32)state / 2^31."""
    state = seed

    def next_f(n):
        nonlocal state
        out = np.empty(n, np.float32)
        for i in range(n):
            state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
            s = state - (1 << 32) if state >= (1 << 31) else state
            out[i] = np.float32(s) * np.float32(1.0 / 2147483648.0)
        return out
    return next_f


def lcg_bf16(vals: np.ndarray) -> np.ndarray:
    """rng_bf16 of tests/test_kernels.c:33-37: (value * 0.1f), truncated to bf16."""
    f = (vals.astype(np.float32) * np.float32(0.1)).astype(np.float32)
    return (f.view(np.uint32) >> 16).astype(np.uint16)


def mel_batch(seconds, seed: int, n_mels: int = 128):
    """Zero-padded [B, n_mels, T_mel_max] batch of N(0,1) log-mel."""
    T_mel = np.array([ctb.t_mel_of_seconds(s) for s in seconds], np.int32)
    T_max = int(T_mel.max())
    mel = np.zeros((len(seconds), n_mels, T_max), np.float32)
    for b, t in enumerate(T_mel):
        rng = np.random.default_rng([seed, b])
        mel[b, :, :t] = rng.standard_normal((n_mels, int(t)), dtype=np.float32)
    return mel, T_mel


def tiny_e2e_case():
    """Configuration 1: 4 utterances, EOS forced at 8-64 tokens.  Lengths are
    drawn from 2-6.5 s instead of 2-8 s: the reference CPU backend's attention
    scratch (backends/cpu/backend.c:247-255) places attn_out T*ENC_D floats
    after the score rows, which need T*(3T-1), so for 3T-1 > ENC_D the two
    overlap and the reference corrupts its own output.  At the tiny width
    (ENC_D 256) that starts at T_enc 86 (about 6.8 s); at full width (1280) at
    T_enc 428 (about 34 s, beyond the reference's 30 s auto-chunking)."""
    rng = np.random.default_rng(101)
    secs = np.round(rng.uniform(2.0, 6.5, 4), 2)
    mel, T_mel = mel_batch(secs, seed=102)
    forced = rng.integers(8, 65, 4).astype(np.int32)
    return dict(weight_seed=1, seconds=secs, mel=mel, T_mel=T_mel, T_mel_max=int(mel.shape[2]),
                forced_len=forced, prompt=np.array(ctb.PROMPT_TINY, np.int32))


def full_decode_case():
    """Full-size decoder slice: 2 sequences, T_enc 26 and 63 (2 s and 5 s)."""
    rng = np.random.default_rng(201)
    T_enc = np.array([26, 63], np.int32)
    enc = np.zeros((2, int(T_enc.max()), 1024), np.float32)
    for b, t in enumerate(T_enc):
        enc[b, :t] = rng.standard_normal((int(t), 1024), dtype=np.float32)
    return dict(weight_seed=0, enc_h=enc, T_enc=T_enc, forced_len=np.array([6, 9], np.int32),
                prompt=np.array(ctb.PROMPT_FULL, np.int32))


def ragged_decode_case(B: int, seed: int, t_lo=5.0, t_hi=30.0, l_lo=20, l_hi=220, enc_std=1.0):
    """Configuration 3 shape: utterances U(t_lo, t_hi) s -> T_enc, EOS forced at
    U{l_lo..l_hi} generated tokens; encoder outputs N(0, enc_std^2)."""
    rng = np.random.default_rng(seed)
    secs = rng.uniform(t_lo, t_hi, B)
    T_enc = np.array([ctb.t_enc_of(ctb.t_mel_of_seconds(s)) for s in secs], np.int32)
    forced = rng.integers(l_lo, l_hi + 1, B).astype(np.int32)
    return dict(seconds=secs, T_enc=T_enc, forced_len=forced, enc_seed=seed + 1, enc_std=enc_std)


def enc_outputs(T_enc, seed: int, d: int = 1024, std: float = 1.0) -> np.ndarray:
    """[B, max(T_enc), d] float32, row-padded with zeros."""
    T_enc = np.asarray(T_enc)
    enc = np.zeros((len(T_enc), int(T_enc.max()), d), np.float32)
    for b, t in enumerate(T_enc):
        rng = np.random.default_rng([seed, b])
        enc[b, :t] = rng.standard_normal((int(t), d), dtype=np.float32) * np.float32(std)
    return enc


def audio(seconds: float, seed: int) -> np.ndarray:
    """Seeded 16 kHz test signal: a few tones plus white noise, float32."""
    n = int(round(seconds * 16000))
    rng = np.random.default_rng(seed)
    t = np.arange(n, dtype=np.float64) / 16000.0
    x = np.zeros(n)
    for f, a in zip(rng.uniform(80.0, 4000.0, 4), rng.uniform(0.05, 0.3, 4)):
        x += a * np.sin(2 * np.pi * f * t + rng.uniform(0, 2 * np.pi))
    x += 0.02 * rng.standard_normal(n)
    return x.astype(np.float32)


def mel_case():
    """Front-end fixture inputs: lengths with and without a partial last hop."""
    return [(seconds, 900 + i) for i, seconds in enumerate((1.0, 2.3456, 0.37))]


def speech_like(seconds: float, seed: int) -> np.ndarray:
    """Seeded 16 kHz signal of tone bursts (0.6-6 s) separated by near-silent
    gaps (0.05-0.8 s, noise floor 1e-3): long-form chunking test input."""
    rng = np.random.default_rng(seed)
    n = int(round(seconds * 16000))
    x = (rng.standard_normal(n) * 1e-3).astype(np.float64)
    t = 0
    while t < n:
        burst = int(rng.uniform(0.6, 6.0) * 16000)
        e = min(n, t + burst)
        tt = np.arange(e - t) / 16000.0
        f = rng.uniform(100.0, 3000.0)
        x[t:e] += rng.uniform(0.05, 0.3) * np.sin(2 * np.pi * f * tt) + 0.02 * rng.standard_normal(e - t)
        t = e + int(rng.uniform(0.05, 0.8) * 16000)
    return x.astype(np.float32)


def longform_case():
    """(seconds, seed, silence_db, silence_dur, target_sec) of the long-form split fixtures."""
    nan = float("nan")
    return [(45.0, 1201, nan, 0.2, 20.0), (130.0, 1202, nan, 0.2, 20.0), (75.5, 1203, -40.0, 0.3, 12.0),
            (61.0, 1204, nan, 0.5, 30.0)]
