"""Audio files in, transcripts out: the reference's file front door.

Host side of load_audio (transcribe.c:124-173), the vocabulary and
print_tokens (:216-262), do_transcribe_file (:990-1030) and the input-folder /
watch mode (:1108-1228), on the engine.

load_audio(path) returns float32 mono samples at 16 kHz.  With `ffmpeg` on
PATH it runs the reference's command (`ffmpeg -i path -f f32le -ar 16000 -ac
1 pipe:1`).  Without it, RIFF/WAVE files are decoded here: PCM 8/16/24/32-bit
and IEEE float 32/64 samples, channels averaged to mono, resampled to 16 kHz
with a polyphase filter when the file's rate differs (ffmpeg's resampler is
not reproduced, so only 16 kHz files give the samples ffmpeg would).

Vocabulary: convert.py's vocab.txt, one SentencePiece piece per line.
`detokenize` follows print_tokens: ids outside the vocabulary and "<|...|>"
specials are skipped, U+2581 becomes a space except before the first
character written, and the line ends with a newline.

`transcribe_files` decodes every file as one packed workload: files up to
30 s in one pass, longer ones chunked at silences with carried context
(do_transcribe_file's rule, through longform.LongFormScheduler), all files'
chunks sharing the engine's batch.  `run_folder` is the input-folder mode:
non-hidden entries in name order, non-audio skipped, `<output>/<stem>.txt`
per file, files whose output exists skipped; with `watch` it then keeps
polling the folder for new files (the reference waits on inotify
IN_CLOSE_WRITE / IN_MOVED_TO; a file here counts as complete once its size
and modification time hold still across one poll) until `stop()` is true.
"""
from __future__ import annotations

import math
import os
import shutil
import struct
import subprocess
import time

import numpy as np

SR = 16000
LONG_S = 30.0          # do_transcribe_file: chunked mode above 30 s
SPACE = "▁"


class AudioError(RuntimeError):
    pass


# ---- decoding ------------------------------------------------------------------

def _read_wav(path: str):
    """(samples [frames, channels] float64 in [-1, 1), rate) of a RIFF/WAVE file."""
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 12 or data[:4] != b"RIFF" or data[8:12] != b"WAVE":
        raise AudioError(f"{path}: not a RIFF/WAVE file")
    fmt = None
    body = None
    pos = 12
    while pos + 8 <= len(data):
        cid, size = data[pos:pos + 4], struct.unpack("<I", data[pos + 4:pos + 8])[0]
        chunk = data[pos + 8:pos + 8 + size]
        if cid == b"fmt ":
            fmt = chunk
        elif cid == b"data":
            body = chunk
        pos += 8 + size + (size & 1)
    if fmt is None or body is None or len(fmt) < 16:
        raise AudioError(f"{path}: missing fmt or data chunk")
    tag, ch, rate, _, align, bits = struct.unpack("<HHIIHH", fmt[:16])
    if tag == 0xFFFE and len(fmt) >= 26:            # WAVE_FORMAT_EXTENSIBLE: the sub-format's tag
        tag = struct.unpack("<H", fmt[24:26])[0]
    if ch < 1 or align != ch * (bits // 8):
        raise AudioError(f"{path}: unsupported layout ({ch} channels, {bits} bits, block {align})")
    n = len(body) // align
    raw = body[:n * align]
    if tag == 1 and bits == 8:
        x = (np.frombuffer(raw, np.uint8).astype(np.float64) - 128.0) / 128.0
    elif tag == 1 and bits == 16:
        x = np.frombuffer(raw, "<i2").astype(np.float64) / 32768.0
    elif tag == 1 and bits == 24:
        b = np.frombuffer(raw, np.uint8).reshape(-1, 3).astype(np.int32)
        v = b[:, 0] | (b[:, 1] << 8) | (b[:, 2] << 16)
        x = np.where(v >= 1 << 23, v - (1 << 24), v).astype(np.float64) / float(1 << 23)
    elif tag == 1 and bits == 32:
        x = np.frombuffer(raw, "<i4").astype(np.float64) / float(1 << 31)
    elif tag == 3 and bits in (32, 64):
        x = np.frombuffer(raw, "<f4" if bits == 32 else "<f8").astype(np.float64)
    else:
        raise AudioError(f"{path}: unsupported sample format (tag {tag}, {bits} bits)")
    return x.reshape(n, ch), int(rate)


def _resample(x: np.ndarray, rate: int) -> np.ndarray:
    if rate == SR:
        return x
    from scipy.signal import resample_poly
    g = math.gcd(SR, rate)
    return resample_poly(x, SR // g, rate // g)


def load_audio(path: str, use_ffmpeg: bool | None = None) -> np.ndarray:
    """float32 mono samples at 16 kHz (transcribe.c:124-173)."""
    if use_ffmpeg is None:
        use_ffmpeg = shutil.which("ffmpeg") is not None
    if use_ffmpeg:
        r = subprocess.run(["ffmpeg", "-hide_banner", "-loglevel", "error", "-i", path, "-f", "f32le", "-ar",
                            str(SR), "-ac", "1", "pipe:1"], stdout=subprocess.PIPE, stderr=subprocess.PIPE)
        if r.returncode != 0:
            raise AudioError(f"ffmpeg failed for: {path}")
        return np.frombuffer(r.stdout, "<f4").copy()
    x, rate = _read_wav(path)
    mono = x.mean(axis=1)
    return _resample(mono, rate).astype(np.float32)


def is_audio(path: str) -> bool:
    """Whether the file decodes as audio (the reference asks ffprobe; without
    it, a RIFF/WAVE header with a readable format is the test)."""
    if not os.path.isfile(path):
        return False
    if shutil.which("ffprobe"):
        r = subprocess.run(["ffprobe", "-v", "error", "-select_streams", "a:0", "-show_entries", "stream=codec_type",
                            "-of", "csv=p=0", path], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL)
        return r.returncode == 0 and b"audio" in r.stdout
    try:
        _read_wav(path)
        return True
    except (AudioError, OSError, ValueError):
        return False


# ---- vocabulary -----------------------------------------------------------------

def load_vocab(path: str) -> list:
    """convert.py's vocab.txt: piece i on line i."""
    with open(path, encoding="utf-8") as f:
        return f.read().split("\n")


def detokenize(tokens, vocab: list) -> str:
    """print_tokens (transcribe.c:240-262) as a string, newline included."""
    out, any_ = [], False
    for t in tokens:
        t = int(t)
        if t < 0 or t >= len(vocab):
            continue
        piece = vocab[t]
        if piece.startswith("<|"):
            continue
        for c in piece:
            if c == SPACE:
                if any_:
                    out.append(" ")
            else:
                out.append(c)
            any_ = True
    return "".join(out) + "\n"


# ---- transcription --------------------------------------------------------------

def transcribe_files(engine, samples_list, prompt, forced_len=None, silence_db: float = math.nan,
                     silence_dur: float = 0.2, target_sec: float = 20.0, chunk: bool = False) -> list:
    """Generated tokens per chunk for each input, all inputs sharing the engine:
    [[tokens of chunk 0, ...] per input].  An input longer than 30 s, or every
    input with `chunk`, is cut at silences (transcribe_file_chunked); shorter
    ones run in one pass (transcribe_chunk)."""
    from importlib import import_module
    lf = import_module(__package__ + ".longform")
    sched = lf.LongFormScheduler(engine, prompt, forced_len=forced_len, silence_db=silence_db,
                                 silence_dur=silence_dur, target_sec=target_sec)
    for i, x in enumerate(samples_list):
        sched.add(i, x, single=not chunk and len(x) <= int(SR * LONG_S))
    out = sched.run()
    return [out[i] for i in range(len(samples_list))]


def _stem(name: str) -> str:
    dot = name.rfind(".")
    return name[:dot] if dot > 0 else name


def run_folder(engine, input_folder: str, output_folder: str, vocab: list, prompt, watch: bool = False,
               poll_s: float = 1.0, stop=None, chunk: bool = False, **opts) -> list:
    """The input-folder mode (transcribe.c:1108-1228): transcribe every audio
    file of input_folder not yet transcribed into output_folder/<stem>.txt,
    one line per chunk.  The files found at one scan go to the engine as one
    workload.  Returns the output paths written, in order."""
    written = []
    seen = {}

    def scan(initial: bool):
        todo = []
        for n in sorted(x for x in os.listdir(input_folder) if not x.startswith(".")):
            path = os.path.join(input_folder, n)
            out = os.path.join(output_folder, _stem(n) + ".txt")
            if os.path.exists(out) or not os.path.isfile(path):
                continue
            if not initial:
                # a file that appeared while watching is taken once its size and
                # modification time held still across one poll (written and closed)
                st = os.stat(path)
                sig = (st.st_size, st.st_mtime_ns)
                if seen.get(path) != sig:
                    seen[path] = sig
                    continue
            if is_audio(path):
                todo.append((path, out))
        return todo

    def process(todo):
        if not todo:
            return
        xs = [load_audio(p) for p, _ in todo]
        res = transcribe_files(engine, xs, prompt, chunk=chunk, **opts)
        for (_, out), chunks in zip(todo, res):
            with open(out, "w", encoding="utf-8") as f:
                for toks in chunks:
                    f.write(detokenize(toks, vocab))
            written.append(out)

    process(scan(True))
    while watch and not (stop and stop()):
        time.sleep(poll_s)
        process(scan(False))
    return written
