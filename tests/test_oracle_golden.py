"""Pin the CPU oracle (oracle/oracle.c) to the reference.

1. The reference's own kernel test vectors (tests/test_kernels.c of the
   reference on its CPU backend, tests/golden/test_kernels_ref_cpu.bin).
2. The reference CPU backend itself (oracle/_ref/libref_cpu.so), function by
   function on seeded inputs -- bit-exact (same arithmetic order, same flags).
3. End to end: configuration 1 (tiny model, log-mel -> tokens) and a full-size
   decoder slice, against fixtures produced by the reference's model.h.
4. The log-mel front-end against the reference's compute_mel.
"""
import ctypes
import os

import numpy as np
import pytest

import inputs
import pyoracle as po

FULL = None


def _full(wmod):
    global FULL
    if FULL is None:
        FULL = dict(wmod.FULL_DIMS)
    return FULL


# ---------------------------------------------------------------- 1 ----------

def test_kernels_golden_vectors(wmod):
    """Replays tests/test_kernels.c (reference) input generation and checks the
    oracle's results against the reference CPU backend's recorded output."""
    gold = np.fromfile(po.os.path.join(po.os.path.dirname(inputs.__file__), "test_kernels_ref_cpu.bin"),
                       dtype=np.float32)
    L = po.lib()
    d = po.dims_struct(_full(wmod))
    rng = inputs.lcg_stream()
    blob = inputs.lcg_bf16(rng(64 + 64 + 128 * 64 + 128))
    ln_w, ln_b = blob[0:64], blob[64:128]
    lin_W, lin_b = blob[128:128 + 8192], blob[8320:8448]
    out = []
    src = rng(8 * 64)
    dst = np.zeros_like(src)
    L.orc_layernorm(po.fp(dst), po.fp(src), ln_w.ctypes.data, ln_b.ctypes.data, 8, 64)
    out.append(dst)
    for ep in (0, 1, 2):
        x = rng(4 * 64)
        y = np.zeros(4 * 128, np.float32)
        L.orc_linear(po.fp(y), po.fp(x), lin_W.ctypes.data, lin_b.ctypes.data, 4, 64, 128, ep, 0.0)
        out.append(y)
    x = rng(4 * 64)
    acc = rng(4 * 128)
    L.orc_linear(po.fp(acc), po.fp(x), lin_W.ctypes.data, lin_b.ctypes.data, 4, 64, 128, 3, 0.5)
    out.append(acc)
    pairs = rng(512)
    dsta, srca = pairs[0::2].copy(), pairs[1::2].copy()
    L.orc_add_inplace(po.fp(dsta), po.fp(srca), 256)
    out.append(dsta)
    mask = np.zeros(64, np.float32)
    L.orc_fill_causal_mask(po.fp(mask), 8)
    out.append(mask)
    pe = np.zeros(7 * 1280, np.float32)
    L.orc_make_rel_pos_emb(ctypes.byref(d), po.fp(pe), 4)
    out.append(pe)
    q = (rng(4 * 1024) * np.float32(0.1)).astype(np.float32)
    k = (rng(6 * 1024) * np.float32(0.1)).astype(np.float32)
    v = rng(6 * 1024)
    o = np.zeros(4 * 1024, np.float32)
    L.orc_sdp_attn(ctypes.byref(d), po.fp(o), po.fp(q), po.fp(k), po.fp(v), po.null_f(), 4, 6)
    out.append(o)
    mine = np.concatenate(out)
    assert mine.shape == gold.shape
    err = np.abs(mine - gold)
    # the reference's own tolerance is 1e-4 absolute (tests/run_tests.sh:12)
    assert err.max() <= 1e-6, f"max abs err {err.max()} at {err.argmax()}"


# ---------------------------------------------------------------- 2 ----------

_f = ctypes.POINTER(ctypes.c_float)
_i = ctypes.POINTER(ctypes.c_int)


@pytest.fixture(scope="module")
def reflib():
    L = po.ref_lib("libref_cpu.so")
    if L is None:
        pytest.skip("reference CPU backend not built (oracle/_ref/ needs the reference tree)")
    return L


@pytest.fixture(scope="module")
def small_model(wmod):
    """Full-width weights with one encoder layer (keeps generation fast)."""
    dims = dict(wmod.FULL_DIMS, enc_n=1)
    wb = wmod.make_blob(dims, seed=7)
    return wb, wmod.weights_struct(wb)


def _rand(shape, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(scale))


def test_oracle_equals_reference_primitives(reflib, small_model, wmod):
    wb, ws = small_model
    L = po.lib()
    d = po.dims_struct(_full(wmod))
    R = reflib
    L1 = ws.enc[0]
    D0 = ws.dec[0]

    # layernorm / linear family / add
    x = _rand((5, 1280), 1)
    a, b = np.zeros_like(x), np.zeros_like(x)
    R.backend_layernorm(po.fp(a), po.fp(x), ctypes.c_void_p(L1.sa_lnw), ctypes.c_void_p(L1.sa_lnb), 5, 1280)
    L.orc_layernorm(po.fp(b), po.fp(x), L1.sa_lnw, L1.sa_lnb, 5, 1280)
    assert np.array_equal(a, b)
    for ep, fn in enumerate(["backend_linear", "backend_linear_silu", "backend_linear_relu"]):
        a = np.zeros((5, 5120), np.float32)
        b = np.zeros_like(a)
        getattr(R, fn)(po.fp(a), po.fp(x), ctypes.c_void_p(L1.ff1_w1), ctypes.c_void_p(L1.ff1_b1), 5, 1280, 5120)
        L.orc_linear(po.fp(b), po.fp(x), L1.ff1_w1, L1.ff1_b1, 5, 1280, 5120, ep, 0.0)
        assert np.array_equal(a, b), fn
    h = _rand((5, 5120), 2)
    a, b = _rand((5, 1280), 3), _rand((5, 1280), 3)
    R.backend_linear_fmadd(po.fp(a), ctypes.c_float(0.5), po.fp(h), ctypes.c_void_p(L1.ff1_w2),
                           ctypes.c_void_p(L1.ff1_b2), 5, 5120, 1280)
    L.orc_linear(po.fp(b), po.fp(h), L1.ff1_w2, L1.ff1_b2, 5, 5120, 1280, 3, 0.5)
    assert np.array_equal(a, b)

    # relative positions + relative-position MHSA + conv module
    T = 13
    pa = np.zeros((2 * T - 1, 1280), np.float32)
    pb = np.zeros_like(pa)
    R.backend_make_rel_pos_emb(po.fp(pa), T)
    L.orc_make_rel_pos_emb(ctypes.byref(d), po.fp(pb), T)
    assert np.array_equal(pa, pb)
    x = _rand((T, 1280), 4)
    xa, xb = x.copy(), x.copy()
    work = np.zeros(64 * T * 1280 + 4 * T * T, np.float32)
    R.backend_rel_pos_mhsa(po.fp(xa), po.fp(pa), T, ctypes.byref(L1), po.fp(work))
    L.orc_rel_pos_mhsa(ctypes.byref(d), po.fp(xb), po.fp(pb), T, ctypes.addressof(L1))
    assert np.array_equal(xa, xb)
    xa, xb = x.copy(), x.copy()
    R.backend_conformer_conv(po.fp(xa), T, ctypes.byref(L1), po.fp(work))
    L.orc_conformer_conv(ctypes.byref(d), po.fp(xb), T, ctypes.addressof(L1))
    assert np.array_equal(xa, xb)

    # subsampling (ragged: T_mel < stride)
    T_mel, stride = 57, 64
    mel = np.zeros((128, stride), np.float32)
    mel[:, :T_mel] = _rand((128, T_mel), 5)
    T1 = (T_mel + 1) // 2
    T2 = (T1 + 1) // 2
    Te = (T2 + 1) // 2
    xa, xb = np.zeros((Te, 1280), np.float32), np.zeros((Te, 1280), np.float32)
    work = np.zeros(256 * (T1 * 64 + T2 * 32) * 2 + T_mel * 128 + Te * 4096, np.float32)
    R.backend_encoder_subsampling(po.fp(mel), T_mel, stride, po.fp(xa), Te, po.fp(work), ctypes.byref(ws))
    L.orc_encoder_subsampling(ctypes.byref(d), po.fp(mel), T_mel, stride, po.fp(xb), Te, ctypes.addressof(ws))
    assert np.array_equal(xa, xb)

    # decoder attention with a causal mask, embed, LM head
    Tq, Tk = 7, 7
    q, k, v = _rand((Tq, 1024), 6, 0.3), _rand((Tk, 1024), 7, 0.3), _rand((Tk, 1024), 8)
    mask = np.zeros((Tq, Tk), np.float32)
    R.backend_fill_causal_mask(po.fp(mask), Tq)
    oa, ob = np.zeros((Tq, 1024), np.float32), np.zeros((Tq, 1024), np.float32)
    work = np.zeros(Tq * Tk * 8, np.float32)
    R.backend_sdp_attn(po.fp(oa), po.fp(q), po.fp(k), po.fp(v), po.fp(mask), Tq, Tk, po.fp(work))
    L.orc_sdp_attn(ctypes.byref(d), po.fp(ob), po.fp(q), po.fp(k), po.fp(v), po.fp(mask), Tq, Tk)
    assert np.array_equal(oa, ob)
    toks = np.array([13764, 7, 4, 16, 62], np.int32)
    ha, hb = np.zeros((5, 1024), np.float32), np.zeros((5, 1024), np.float32)
    args = [ctypes.c_void_p(ws.etw), ctypes.c_void_p(ws.epw), ctypes.c_void_p(ws.elnw), ctypes.c_void_p(ws.elnb)]
    R.backend_embed(po.fp(ha), po.ip(toks), 5, 3, *args)
    L.orc_embed(ctypes.byref(d), po.fp(hb), po.ip(toks), 5, 3, ws.etw, ws.epw, ws.elnw, ws.elnb)
    assert np.array_equal(ha, hb)
    la, lb = np.zeros(16384, np.float32), np.zeros(16384, np.float32)
    R.backend_lm_head(po.fp(la), po.fp(ha[4]), ctypes.c_void_p(ws.etw), ctypes.c_void_p(ws.hdb))
    L.orc_lm_head(ctypes.byref(d), po.fp(lb), po.fp(hb[4].copy()), ws.etw, ws.hdb)
    assert np.array_equal(la, lb)

    # batched decode helpers (ragged S and T_enc, one inactive item)
    B = 4
    active = np.array([1, 1, 0, 1], np.int32)
    S_dev = np.array([11, 37, 5, 12], np.int32)
    toks = np.array([5, 900, 0, 16000], np.int32)
    ha, hb = np.zeros((B, 1024), np.float32), np.zeros((B, 1024), np.float32)
    R.backend_embed_decode_batch(po.fp(ha), po.ip(toks), po.ip(S_dev), po.ip(active), B, *args)
    L.orc_embed_decode_batch(ctypes.byref(d), po.fp(hb), po.ip(toks), po.ip(S_dev), po.ip(active), B,
                             ws.etw, ws.epw, ws.elnw, ws.elnb)
    assert np.array_equal(ha, hb)
    stride = 40
    ca = np.zeros((B, stride, 1024), np.float32)
    cb = np.zeros_like(ca)
    xin = _rand((B, 1024), 9)
    R.backend_linear_to_kvcache_batch(po.fp(ca), po.fp(xin), ctypes.c_void_p(D0.sa_kw), ctypes.c_void_p(D0.sa_kb),
                                      B, stride, 1024, 1024)
    L.orc_linear_to_kvcache_batch(po.fp(cb), po.fp(xin), D0.sa_kw, D0.sa_kb, B, stride, 1024, 1024, po.ip(S_dev))
    assert np.array_equal(ca, cb)
    K, V = _rand((B, stride, 1024), 10, 0.3), _rand((B, stride, 1024), 11)
    Q = _rand((B, 1024), 12, 0.3)
    oa, ob = np.zeros((B, 1024), np.float32), np.zeros((B, 1024), np.float32)
    work = np.zeros(B * 8 * stride, np.float32)
    R.backend_sdp_attn_batch_decode_sa(po.fp(oa), po.fp(Q), po.fp(K), po.fp(V), stride, B, po.fp(work))
    L.orc_sdp_attn_batch_decode(ctypes.byref(d), po.fp(ob), po.fp(Q), po.fp(K), po.fp(V), stride, B, po.ip(S_dev))
    assert np.array_equal(oa, ob)
    T_enc = np.array([3, 40, 17, 1], np.int32)
    R.backend_upload_T_enc(po.ip(T_enc), B)
    R.backend_sdp_attn_batch_decode_ca(po.fp(oa), po.fp(Q), po.fp(K), po.fp(V), stride, B, po.fp(work))
    L.orc_sdp_attn_batch_decode(ctypes.byref(d), po.fp(ob), po.fp(Q), po.fp(K), po.fp(V), stride, B, po.ip(T_enc))
    assert np.array_equal(oa, ob)
    la, lb = np.zeros((B, 16384), np.float32), np.zeros((B, 16384), np.float32)
    R.backend_lm_head_batch(po.fp(la), po.fp(ha), ctypes.c_void_p(ws.etw), ctypes.c_void_p(ws.hdb), po.ip(active), B)
    L.orc_lm_head_batch(ctypes.byref(d), po.fp(lb), po.fp(hb), ws.etw, ws.hdb, po.ip(active), B)
    assert np.array_equal(la, lb)
    # ties: argmax keeps the lowest index (strict >, backends/cpu/backend.c:452-453)
    la[1, 100] = la[1, 7000] = la[1].max() + 1.0
    oa_i, ob_i = np.full(B, -7, np.int32), np.full(B, -7, np.int32)
    R.backend_argmax_batch(po.ip(oa_i), po.fp(la), po.ip(active), B)
    L.orc_argmax_batch(ctypes.byref(d), po.ip(ob_i), po.fp(la), po.ip(active), B)
    assert np.array_equal(oa_i, ob_i) and oa_i[1] == 100 and oa_i[2] == -7


# ---------------------------------------------------------------- 3 ----------

def test_tiny_config_end_to_end(wmod):
    """Configuration 1 (tiny, fp32, CPU): log-mel -> greedy tokens equals the
    reference model.h + CPU backend run recorded in tiny_e2e_ref.npz."""
    gold = np.load(po.os.path.join(po.os.path.dirname(inputs.__file__), "tiny_e2e_ref.npz"))
    case = inputs.tiny_e2e_case()
    assert np.isclose(case["mel"].astype(np.float64).sum(), float(gold["mel_checksum"]))
    dims = wmod.TINY_DIMS
    wb = wmod.make_blob(dims, seed=case["weight_seed"])
    ws = wmod.weights_struct(wb)
    L = po.lib()
    d = po.dims_struct(dims)
    B = case["mel"].shape[0]
    T_enc = np.array([inputs.ctb.t_enc_of(int(t)) for t in case["T_mel"]], np.int32)
    Tm = int(T_enc.max())
    enc_h = np.zeros((B, Tm, dims["dec_d"]), np.float32)
    L.orc_encoder_forward_batch(ctypes.byref(d), ctypes.addressof(ws), po.fp(case["mel"]), B, case["T_mel_max"],
                                po.ip(case["T_mel"]), po.ip(T_enc), Tm, po.fp(enc_h))
    for b in range(B):
        assert np.array_equal(enc_h[b, :T_enc[b]], gold["enc_h"][b, :T_enc[b]])
    tokens, n_tok, am, mg = po.decode_batch(dims, ws, enc_h, T_enc, case["prompt"], case["forced_len"])
    assert np.array_equal(n_tok, gold["n_tok"])
    assert np.array_equal(tokens, gold["tokens"])
    sel = ~np.isnan(gold["margin"])
    assert np.array_equal(mg[sel], gold["margin"][sel])


def test_full_decoder_slice(wmod):
    """Full-size decoder (prefill + batched decode, two ragged sequences)
    equals the reference model.h + CPU backend run in full_decode_ref.npz."""
    gold = np.load(po.os.path.join(po.os.path.dirname(inputs.__file__), "full_decode_ref.npz"))
    case = inputs.full_decode_case()
    assert np.isclose(case["enc_h"].astype(np.float64).sum(), float(gold["enc_checksum"]))
    wb = wmod.make_blob(wmod.FULL_DIMS, seed=case["weight_seed"], parts=("dec",))
    ws = wmod.weights_struct(wb)
    tokens, n_tok, am, mg = po.decode_batch(wmod.FULL_DIMS, ws, case["enc_h"], case["T_enc"], case["prompt"],
                                            case["forced_len"])
    assert np.array_equal(n_tok, gold["n_tok"])
    assert np.array_equal(tokens, gold["tokens"])
    sel = ~np.isnan(gold["margin"])
    np.testing.assert_allclose(mg[sel], gold["margin"][sel], rtol=0, atol=1e-5)


def test_mel_front_end_matches_reference():
    """The oracle's log-mel front-end equals the reference's compute_mel
    (transcribe.c:177-214), recorded in tests/golden/mel_ref.npz from the
    reference built here; and, when that build is present, on fresh lengths."""
    gold = np.load(os.path.join(os.path.dirname(inputs.__file__), "mel_ref.npz"))
    for k, (seconds, seed) in enumerate(inputs.mel_case()):
        x = inputs.audio(seconds, seed)
        assert np.float64(x.astype(np.float64).sum()) == gold[f"checksum{k}"]
        assert np.array_equal(po.compute_mel(x), gold[f"mel{k}"]), k
    path = os.path.join(po.REF_DIR, "libref_mel.so")
    if os.path.exists(path):
        R = ctypes.CDLL(path)
        R.refmel_compute.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        for n in (160, 159, 31999, 80000):
            x = inputs.audio(n / 16000.0, n)
            ref = np.zeros((128, 1 + n // 160), np.float32)
            R.refmel_compute(x.ctypes.data, len(x), ref.ctypes.data)
            # one frame (n < 160): the unbiased variance divides by T - 1 = 0 and
            # the reference yields NaN; the oracle reproduces it
            assert np.array_equal(po.compute_mel(x), ref, equal_nan=True), n


def test_full_size_encoder_matches_live_reference(wmod):
    """Full-size encoder (48 Conformer layers at width 1280, model.h dims) plus a
    short greedy decode: the oracle's orc_encoder_forward_batch and decoder give
    the same encoder rows and tokens, bit for bit, as the reference's own
    model.h encoder_forward_batch + decode loop on its CPU backend
    (oracle/_ref/libref_decode_cpu.so, built from the reference sources).  Two
    short ragged utterances keep the reference's single-threaded run to
    seconds; the arithmetic per row is the one every length uses."""
    L = po.ref_lib("libref_decode_cpu.so")
    if L is None:
        pytest.skip("reference decode harness not built (oracle/_ref/ needs the reference tree)")
    L = po.bind_ref_decode(L)
    dims = wmod.FULL_DIMS
    wb = wmod.make_blob(dims, seed=11)
    ws = wmod.weights_struct(wb)
    secs = [0.6, 0.35]
    mel, T_mel = inputs.mel_batch(secs, seed=907)
    B, T_mel_max = mel.shape[0], mel.shape[2]
    T_enc = np.array([inputs.ctb.t_enc_of(int(t)) for t in T_mel], np.int32)
    Tm = inputs.ctb.t_enc_of(T_mel_max)
    prompt = np.array(inputs.ctb.PROMPT_FULL, np.int32)
    forced = np.array([5, 4], np.int32)

    L.refh_bind_weights(ctypes.addressof(ws))
    L.backend_init(0)
    r_tok = np.zeros((B, 1024), np.int32)
    r_n = np.zeros(B, np.int32)
    r_am = np.full((B, 1024), -1, np.int32)
    r_mg = np.full((B, 1024), np.nan, np.float32)
    r_enc = np.zeros((B, Tm, dims["dec_d"]), np.float32)
    L.refh_transcribe_batch(B, po.fp(mel), T_mel_max, po.ip(T_mel), po.ip(prompt), len(prompt), po.ip(forced),
                            po.null_i(), po.ip(r_tok), po.ip(r_n), po.ip(r_am), po.fp(r_mg), po.fp(r_enc))
    L.backend_thread_cleanup()

    O = po.lib()
    d = po.dims_struct(dims)
    o_enc = np.zeros((B, Tm, dims["dec_d"]), np.float32)
    O.orc_encoder_forward_batch(ctypes.byref(d), ctypes.addressof(ws), po.fp(mel), B, T_mel_max, po.ip(T_mel),
                                po.ip(T_enc), Tm, po.fp(o_enc))
    for b in range(B):
        assert np.array_equal(o_enc[b, :T_enc[b]], r_enc[b, :T_enc[b]]), f"encoder rows of utterance {b}"
    tokens, n_tok, am, mg = po.decode_batch(dims, ws, o_enc, T_enc, prompt, forced)
    assert np.array_equal(n_tok, r_n)
    assert np.array_equal(tokens, r_tok)
    sel = ~np.isnan(r_mg)
    assert np.array_equal(mg[sel], r_mg[sel])
