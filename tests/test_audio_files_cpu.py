"""Audio-file front door (cohere-transcribe_b200/audio_files.py) on CPU: WAV
decoding, the vocabulary printer, and the input-folder / watch mode driven
against a stand-in engine (transcribe.c:124-173, :216-262, :990-1030,
:1108-1228)."""
import importlib
import os
import struct
import threading
import time
import wave

import numpy as np

af = importlib.import_module("cohere-transcribe_b200.audio_files")


def write_wav_pcm16(path, x, rate=16000, channels=1):
    a = np.clip(np.round(np.asarray(x) * 32768.0), -32768, 32767).astype("<i2")
    with wave.open(str(path), "wb") as w:
        w.setnchannels(channels)
        w.setsampwidth(2)
        w.setframerate(rate)
        w.writeframes(a.tobytes())


def write_wav_raw(path, payload: bytes, tag: int, channels: int, rate: int, bits: int):
    align = channels * bits // 8
    fmt = struct.pack("<HHIIHH", tag, channels, rate, rate * align, align, bits)
    body = b"fmt " + struct.pack("<I", len(fmt)) + fmt + b"data" + struct.pack("<I", len(payload)) + payload
    with open(path, "wb") as f:
        f.write(b"RIFF" + struct.pack("<I", 4 + len(body)) + b"WAVE" + body)


def test_pcm16_stereo_is_averaged_to_mono(tmp_path):
    rng = np.random.default_rng(1)
    st = rng.integers(-30000, 30000, size=(1600, 2)).astype(np.int16)
    write_wav_pcm16(tmp_path / "s.wav", st.reshape(-1) / 32768.0, channels=2)
    got = af.load_audio(str(tmp_path / "s.wav"), use_ffmpeg=False)
    want = ((st[:, 0].astype(np.float64) + st[:, 1]) / 2 / 32768.0).astype(np.float32)
    assert got.dtype == np.float32 and np.array_equal(got, want)


def test_float32_pcm24_pcm8(tmp_path):
    x = np.linspace(-0.9, 0.9, 480).astype(np.float32)
    write_wav_raw(tmp_path / "f.wav", x.astype("<f4").tobytes(), 3, 1, 16000, 32)
    assert np.array_equal(af.load_audio(str(tmp_path / "f.wav"), use_ffmpeg=False), x)
    v = np.array([-(1 << 23), -1, 0, 1, (1 << 23) - 1], np.int64)
    b = np.stack([(v & 0xFF), (v >> 8) & 0xFF, (v >> 16) & 0xFF], 1).astype(np.uint8).tobytes()
    write_wav_raw(tmp_path / "p24.wav", b, 1, 1, 16000, 24)
    assert np.array_equal(af.load_audio(str(tmp_path / "p24.wav"), use_ffmpeg=False),
                          (v / float(1 << 23)).astype(np.float32))
    write_wav_raw(tmp_path / "p8.wav", bytes([0, 128, 255]), 1, 1, 16000, 8)
    assert np.array_equal(af.load_audio(str(tmp_path / "p8.wav"), use_ffmpeg=False),
                          np.array([-1.0, 0.0, 127 / 128], np.float32))


def test_other_rates_are_resampled(tmp_path):
    t8 = np.arange(8000) / 8000.0
    write_wav_pcm16(tmp_path / "r8k.wav", 0.5 * np.sin(2 * np.pi * 200.0 * t8), rate=8000)
    got = af.load_audio(str(tmp_path / "r8k.wav"), use_ffmpeg=False)
    assert len(got) == 16000
    t16 = np.arange(16000) / 16000.0
    mid = slice(2000, 14000)   # away from the filter's edges
    assert np.max(np.abs(got[mid] - 0.5 * np.sin(2 * np.pi * 200.0 * t16[mid]))) < 1e-2


def test_is_audio(tmp_path, monkeypatch):
    monkeypatch.setattr(af.shutil, "which", lambda name: None)
    write_wav_pcm16(tmp_path / "a.wav", np.zeros(160))
    (tmp_path / "notes.txt").write_text("hello")
    assert af.is_audio(str(tmp_path / "a.wav"))
    assert not af.is_audio(str(tmp_path / "notes.txt"))
    assert not af.is_audio(str(tmp_path / "missing.wav"))


def test_detokenize_follows_print_tokens():
    vocab = ["<|endoftext|>", "▁hello", "▁wor", "ld", ",", "<|pnc|>", "▁▁x"]
    assert af.detokenize([1, 2, 3, 4, 0], vocab) == "hello world,\n"
    assert af.detokenize([5, 3, 1, 99, -1], vocab) == "ld hello\n"
    assert af.detokenize([6], vocab) == " x\n"          # the first U+2581 writes nothing, the second a space
    assert af.detokenize([], vocab) == "\n"


class FakeEngine:
    """Stand-in for abi.Engine: every utterance decodes to [len(samples) % 5 + 1, EOS]
    (EOS = 0 here) and finishes on the next step."""

    def __init__(self):
        self.pending, self.done, self.prompts, self.submitted = {}, {}, [], []

    def set_prompt(self, p):
        self.prompts.append(None if p is None else list(p))

    def submit_audio(self, uid, x, forced):
        self.submitted.append((uid, len(x)))
        self.pending[uid] = np.array([len(x) % 5 + 1, 0], np.int32)

    def step(self, n):
        self.done.update(self.pending)
        self.pending = {}

    def poll(self):
        d, self.done = self.done, {}
        return d


VOCAB = ["<|endoftext|>", "▁a", "▁b", "▁c", "▁d", "▁e"]


def test_run_folder_initial_scan(tmp_path):
    src, dst = tmp_path / "in", tmp_path / "out"
    src.mkdir(); dst.mkdir()
    write_wav_pcm16(src / "b.wav", np.zeros(16001))
    write_wav_pcm16(src / "a.wav", np.zeros(16002))
    write_wav_pcm16(src / ".hidden.wav", np.zeros(16003))
    (src / "readme.txt").write_text("not audio")
    write_wav_pcm16(src / "done.wav", np.zeros(16004))
    (dst / "done.txt").write_text("already transcribed\n")
    eng = FakeEngine()
    out = af.run_folder(eng, str(src), str(dst), VOCAB, prompt=[7] * 10)
    assert [os.path.basename(p) for p in out] == ["a.txt", "b.txt"]
    assert (dst / "a.txt").read_text() == af.detokenize([16002 % 5 + 1, 0], VOCAB)
    assert (dst / "b.txt").read_text() == af.detokenize([16001 % 5 + 1, 0], VOCAB)
    assert (dst / "done.txt").read_text() == "already transcribed\n"
    assert sorted(n for _, n in eng.submitted) == [16001, 16002]


def test_long_file_is_chunked(tmp_path):
    src, dst = tmp_path / "in", tmp_path / "out"
    src.mkdir(); dst.mkdir()
    rng = np.random.default_rng(3)
    speech = lambda s: 0.3 * rng.standard_normal(int(16000 * s))
    quiet = lambda s: 0.001 * rng.standard_normal(int(16000 * s))
    # 36 s with three 1 s pauses (the automatic threshold sits 20 dB above the
    # quietest 5% of frames)
    x = np.concatenate([speech(10.0), quiet(1.0), speech(10.0), quiet(1.0), speech(10.0), quiet(1.0), speech(3.0)])
    write_wav_pcm16(src / "long.wav", x)
    eng = FakeEngine()
    af.run_folder(eng, str(src), str(dst), VOCAB, prompt=list(range(10)))
    lines = (dst / "long.txt").read_text().splitlines()
    assert len(lines) == len(eng.submitted) >= 2            # one line per chunk
    assert sum(n for _, n in eng.submitted) == len(x)
    # the second chunk's prompt carries the first chunk's text (its token, EOS dropped)
    carried = [p for p in eng.prompts if p is not None][1]
    assert carried[:2] == [0, 1] and carried[2] == eng.submitted[0][1] % 5 + 1


def test_watch_picks_up_new_files(tmp_path):
    src, dst = tmp_path / "in", tmp_path / "out"
    src.mkdir(); dst.mkdir()
    write_wav_pcm16(src / "first.wav", np.zeros(16000))
    eng = FakeEngine()
    result = {}

    def run():
        result["out"] = af.run_folder(eng, str(src), str(dst), VOCAB, prompt=[7] * 10, watch=True, poll_s=0.05,
                                      stop=lambda: (dst / "second.txt").exists())

    th = threading.Thread(target=run)
    th.start()
    deadline = time.time() + 10
    while not (dst / "first.txt").exists() and time.time() < deadline:
        time.sleep(0.02)
    write_wav_pcm16(src / "second.wav", np.zeros(8000))
    th.join(timeout=10)
    assert not th.is_alive()
    assert [os.path.basename(p) for p in result["out"]] == ["first.txt", "second.txt"]
