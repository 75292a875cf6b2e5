"""CPU check of bench.py's output contract (no GPU).

bench.py's host logic -- workload generation, leg timing, the roofline and
traffic arithmetic, the configuration-2 summary, the reference arm's line --
runs here against a stand-in engine that returns fixed device times, so the
JSON line a driver parses keeps its keys and units.  The numbers are the
stand-in's; the real measurement needs a B200.
"""
import importlib
import json
import sys

import numpy as np
import pytest

REQUIRED = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
            "vs_baseline", "dtype", "data", "config", "e2e", "gpu_launches", "roofline", "clocks")


@pytest.fixture()
def bench_mod(monkeypatch):
    bench = importlib.import_module("bench")
    abi = importlib.import_module("cohere-transcribe_b200.abi")
    W = importlib.import_module("cohere-transcribe_b200.weights")

    class Blob:
        nbytes = 0

        def ptr(self):
            return 0

    class StandInEngine:
        """Fixed device times: 1 ms per leg for steps / admission / encoder."""

        def __init__(self, lib, dev, wb, ws, profile=0, **kw):
            self.q, self.times, self.rep = {}, [], {}
            self.st = {f: 0.0 for f, _ in abi.EngineStats._fields_}

        def submit(self, i, x, f):
            self.q[i] = int(f)

        submit_audio = submit

        def submit_mel(self, i, x, f):
            assert x.shape[0] == 128
            self.q[i] = int(f)

        def step(self, n):   # the stand-in finishes everything it holds at once
            return 0

        def encode(self, m):
            return m

        def log_mel(self, a):
            return a

        def run(self):
            for k in ("step_ms", "admit_ms", "enc_ms", "cross_attn_ms", "self_attn_ms", "ffn_ms"):
                self.st[k] += 1.0
            for k in ("cross_kv_bytes", "self_kv_bytes", "ffn_bytes"):
                self.st[k] += 1e9
            self.st["steps"] += 10
            self.st["kernel_launches"] += 700
            self.times += [0.5] * 10
            n = self.rep.get("enc_gemm_ffn1", [0.0, 0])
            self.rep = {"enc_gemm_ffn1": [n[0] + 2.0, n[1] + 96]}

        def step_times(self):
            t = np.array(self.times, np.float32)
            self.times = []
            return t

        def poll(self):
            out = {k: np.zeros(v, np.int32) for k, v in self.q.items()}
            self.q = {}
            return out

        def stats(self):
            return dict(self.st)

        def status(self):
            return 0

        def profile_report(self):
            return dict(self.rep)

        def close(self):
            pass

    class StandInReferenceCUDA:
        """The reference CUDA backend's leg with fixed timings (it needs a GPU)."""

        def __init__(self, ws, case, enc, n):
            self.n = n

        def run(self, wb):
            return {"value": 100.0, "unit": "tokens/s", "kind": "stand-in", "sample": "stand-in",
                    "sample_tokens": 200, "config2": {"tokens_per_s": 50.0, "ms_per_token": 20.0, "sample": "-"}}

    monkeypatch.setattr(bench, "ReferenceCUDA", StandInReferenceCUDA)
    monkeypatch.setattr(W, "make_blob", lambda *a, **k: Blob())
    monkeypatch.setattr(W, "weights_struct", lambda wb: None)
    monkeypatch.setattr(abi, "load", lambda: None)
    monkeypatch.setattr(abi, "Engine", StandInEngine)
    return bench


def _run(bench, capsys, monkeypatch, argv):
    monkeypatch.setattr(sys, "argv", ["bench.py"] + argv)
    bench.main()
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    return json.loads(lines[0])


def test_bench_line_keys_and_units(bench_mod, capsys, monkeypatch):
    d = _run(bench_mod, capsys, monkeypatch, ["--no-cpu", "--steps", "3", "--warmup", "3"])
    for k in REQUIRED:
        assert k in d, k
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True and d["scaling"] == "weak"
    assert set(d["e2e"]) >= {"value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"}
    assert d["e2e"]["h2d_bytes_per_step"] > 0 and d["e2e"]["d2h_bytes_per_step"] > 0
    assert d["gpu_launches"] > 0
    assert d["steps_timed"] > 0 and d["rows_per_step"] is not None
    r = d["roofline"]
    assert set(r) >= {"bound", "achieved", "peak", "unit", "frac", "traffic"}
    assert r["frac"] == pytest.approx(r["achieved"] / r["peak"])
    # the stand-in makes the encoder FFN1 class dominant: its traffic is scaled
    # from the committed capture by packed rows
    assert r["kernel"].startswith("encoder FFN1")
    case, _, _ = bench_mod.workload(0, bench_mod.BATCH)
    rows = float(sum(int(x) for x in case["T_enc"]))
    t = bench_mod.NCU_TRAFFIC[r["kernel"]]
    assert r["traffic"] == pytest.approx(t["bytes"] / t["units"] * rows)
    c2 = d["config2"]
    assert c2["steps_per_run"] == 10 and c2["p50_step_ms"] == pytest.approx(0.5)
    # 3 runs of 200 tokens over 3 x (1 ms admission + 1 ms steps)
    assert c2["decode_tokens_per_s"] == pytest.approx(200 * 3 / 0.006)
    assert d["rtfx"]["unit"] == "audio s / s"
    cb = d["cuda_baseline"]
    assert cb["unit"] == "tokens/s" and cb["value"] == pytest.approx(100.0)
    assert set(cb["config2"]) >= {"tokens_per_s", "ms_per_token"}


def test_reference_arm_line(bench_mod, capsys, monkeypatch):
    class StandInReference:
        def __init__(self, case, enc, audio, n, cap):
            self.sample, self.sample_rtfx = "stand-in", "stand-in"
            self.forced = np.array([40, 60], np.int32)
            self.workload_mean_tokens = 50.0

        def decode(self, warm=False):
            return (4, 0.5) if warm else (100, 2.0)

        def transcribe(self):
            return 8.0, 4.0

    monkeypatch.setattr(bench_mod, "ReferenceCPU", StandInReference)
    d = _run(bench_mod, capsys, monkeypatch, ["--impl", "reference", "--steps", "2", "--warmup", "1"])
    assert d["impl"] == "reference"
    assert d["value"] == pytest.approx(50.0) and d["unit"] == "tokens/s"
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["rtfx"]["value"] == pytest.approx(2.0)
    assert d["cpu_baseline"]["sample_tokens"] == 100 and d["cpu_baseline"]["sample_mean_tokens"] == 50.0


def test_stream_leg_summary(bench_mod, capsys, monkeypatch):
    d = _run(bench_mod, capsys, monkeypatch, ["--no-cpu", "--legs", "S", "--stream-n", "40", "--stream-saturated",
                                              "--steps", "3", "--warmup", "3"])
    c4 = d["config4"]
    assert c4["utterances"] == 40 and c4["workload"].startswith("config 4: 40 utterances")
    assert c4["latency_p50_s"] <= c4["latency_p95_s"] <= c4["latency_max_s"]
    assert c4["generated_tokens"] > 0 and c4["rtfx"] > 0


def test_stream_leg_configuration_5(bench_mod, capsys, monkeypatch):
    d = _run(bench_mod, capsys, monkeypatch, ["--no-cpu", "--legs", "S", "--stream-config", "5", "--stream-n", "30",
                                              "--stream-saturated", "--steps", "3", "--warmup", "3"])
    c5 = d["config5"]
    assert c5["utterances"] == 30 + 704 and "704 windows" in c5["workload"]
