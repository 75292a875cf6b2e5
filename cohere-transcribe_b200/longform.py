"""Long-form transcription: silence-based chunking with carried-over context.

Host side of transcribe_file_chunked (transcribe.c:397-535) on the engine.
A long input is cut at silences: frame RMS over 160-sample hops
(transcribe.c:397-404), an automatic threshold 20 dB above the 5th-percentile
frame RMS (:406-421) or a given level in dB, silence runs of at least
`silence_dur` seconds split at their midpoint (:429-445), and candidate splits
merged so that chunks reach `target_sec` (:455-465).  Chunk c's prompt is the
first two prompt tokens, then the last (at most 64) tokens generated for chunk
c-1 without its EOS, then the rest of the prompt (:509-520, :381-389).  The
chunks of one input are therefore sequential; `LongFormScheduler` keeps many
inputs in flight on one engine, so chunks of different inputs share the packed
decode batch while each input's chunks follow one another.

The arithmetic of the split search is float32 in the reference's order
(sequential sums), so split points equal the reference's on the same samples.
"""
from __future__ import annotations

import math

import numpy as np

SR, HOP = 16000, 160
CARRY_MAX = 64


def frame_rms(samples: np.ndarray) -> np.ndarray:
    """RMS of each full 160-sample hop (transcribe.c:397-404), float32."""
    x = np.asarray(samples, dtype=np.float32)
    n = len(x) // HOP
    f = x[:n * HOP].reshape(n, HOP)
    sq = (f * f).astype(np.float32)
    s = np.cumsum(sq, axis=1, dtype=np.float32)[:, -1] if n else np.zeros(0, np.float32)   # sequential sums
    return np.sqrt(s / np.float32(HOP)).astype(np.float32)


def estimate_silence_thresh(rms: np.ndarray) -> float:
    """20 dB above the 5th-percentile frame RMS, from a 1024-bucket histogram
    (transcribe.c:406-421)."""
    nb = 1024
    b = (rms.astype(np.float32) * np.float32(nb)).astype(np.int64)   # C truncation of a non-negative float
    hist = np.bincount(np.minimum(b, nb - 1), minlength=nb)
    target = len(rms) // 20
    cum = np.cumsum(hist)
    idx = int(np.argmax(cum >= target))
    return float(np.float32(idx) / np.float32(nb) * np.float32(10.0))


def find_splits(rms: np.ndarray, thresh: float, min_silence_sec: float, max_splits: int = 4096) -> list:
    """Sample index of the midpoint of every silence run of at least
    min_silence_sec (transcribe.c:429-445)."""
    min_frames = int(np.float32(min_silence_sec) * np.float32(SR) / np.float32(HOP))
    th = np.float32(thresh)
    out, in_sil, start = [], False, 0
    for f, r in enumerate(rms):
        if r < th:
            if not in_sil:
                start, in_sil = f, True
        elif in_sil:
            if f - start >= min_frames and len(out) < max_splits:
                out.append(((start + f) // 2) * HOP)
            in_sil = False
    return out


def apply_target(splits: list, target_samp: int) -> list:
    """Keep a split only once target_samp samples have accumulated since the
    last kept one (transcribe.c:455-465)."""
    out, prev = [], 0
    for s in splits:
        if s - prev >= target_samp:
            out.append(s)
            prev = s
    return out


def chunk_bounds(samples: np.ndarray, silence_db: float = math.nan, silence_dur: float = 0.2,
                 target_sec: float = 20.0) -> list:
    """[start, end) sample ranges of the chunks (empty ranges dropped), as
    transcribe_file_chunked cuts them (transcribe.c:484-507)."""
    rms = frame_rms(samples)
    if math.isnan(silence_db):
        thresh = estimate_silence_thresh(rms)
    else:
        thresh = float(np.float32(10.0) ** (np.float32(silence_db) / np.float32(20.0)))
    splits = apply_target(find_splits(rms, thresh, silence_dur), int(np.float32(target_sec) * np.float32(SR)))
    out, start = [], 0
    for end in splits + [len(samples)]:
        if end > start:
            out.append((start, end))
        start = end
    return out


def chunk_prompt(prompt: list, carry: list) -> list:
    """prompt[:2] + carry + prompt[2:] (transcribe.c:509-520)."""
    return list(prompt[:2]) + list(carry) + list(prompt[2:])


def carry_of(generated: np.ndarray, cap: int = CARRY_MAX) -> list:
    """The last `cap` generated tokens before the final one (the EOS), as the
    next chunk's context (transcribe.c:381-389)."""
    n = max(len(generated) - 1, 0)
    n = min(n, cap)
    return [int(t) for t in generated[len(generated) - 1 - n:len(generated) - 1]] if n else []


class LongFormScheduler:
    """Transcribe many long inputs on one engine (see the module docstring).

    engine: an abi.Engine with an encoder.  prompt: the base prompt (10
    tokens).  forced_len(chunk_samples) -> int: optional forced EOS length per
    chunk (0 = natural EOS)."""

    def __init__(self, engine, prompt, forced_len=None, silence_db: float = math.nan, silence_dur: float = 0.2,
                 target_sec: float = 20.0, step_block: int = 8):
        self.eng = engine
        self.prompt = list(prompt)
        self.forced_len = forced_len or (lambda n: 0)
        self.opts = (silence_db, silence_dur, target_sec)
        self.step_block = step_block
        self.files = {}

    def add(self, file_id: int, samples: np.ndarray, single: bool = False) -> None:
        """Queue an input; `single` decodes it in one pass (transcribe_chunk)
        instead of cutting it at silences."""
        x = np.ascontiguousarray(samples, dtype=np.float32)
        bounds = [(0, len(x))] if single else chunk_bounds(x, *self.opts)
        self.files[file_id] = {"x": x, "bounds": bounds, "next": 0, "carry": [], "out": []}

    def _submit_next(self, fid: int) -> bool:
        f = self.files[fid]
        c = f["next"]
        if c >= len(f["bounds"]):
            return False
        s, e = f["bounds"][c]
        self.eng.set_prompt(chunk_prompt(self.prompt, f["carry"]))
        self.eng.submit_audio(fid * 65536 + c, f["x"][s:e], self.forced_len(e - s))
        self.eng.set_prompt(None)
        f["next"] = c + 1
        return True

    def run(self) -> dict:
        """{file_id: [generated tokens of each chunk]} once every chunk is done."""
        in_flight = sum(self._submit_next(fid) for fid in self.files)
        while in_flight:
            self.eng.step(self.step_block)
            for uid, toks in self.eng.poll().items():
                fid, c = divmod(int(uid), 65536)
                f = self.files[fid]
                f["out"].append(toks)
                f["carry"] = carry_of(toks)
                in_flight -= 1
                in_flight += self._submit_next(fid)
        return {fid: f["out"] for fid, f in self.files.items()}
