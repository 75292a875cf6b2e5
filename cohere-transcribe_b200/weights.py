"""Seeded random-init weights in the reference's weight-table format.

The reference loads bf16 tensors by their Hugging Face names from one
safetensors blob (model.h:158-225, names from convert.py:58-154) and keeps host
pointers to them in a `Weights` struct (backends/model_types.h:52-77).  There is
no network here, so the real checkpoint is replaced by seeded random weights of
the same names, shapes and dtype (bf16):

  linear / conv weight  N(0, 1/fan_in)        bias          N(0, 0.02)
  LayerNorm / BN gamma  1 + N(0, 0.02)        beta          N(0, 0.02)
  BN running mean       N(0, 0.1)             running var   U(0.5, 1.5)
  token embedding       N(0, 1/sqrt(dec_d))   position table N(0, 0.1)
  pos_bias_u / _v       N(0, 0.02)            LM-head bias  N(0, 0.02)

Each tensor is drawn from its own generator seeded by (seed, crc32(name)), so a
blob that holds only the decoder tensors carries exactly the same decoder
weights as a full blob.
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
import zlib
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field

import numpy as np

# ---- dimensions -----------------------------------------------------------

FULL_DIMS = dict(enc_d=1280, enc_ff=5120, enc_h=8, enc_dk=160, enc_n=48, enc_ck=9, sub_ch=256,
                 dec_d=1024, dec_ff=4096, dec_h=8, dec_dk=128, dec_n=8,
                 vocab=16384, max_seq=1024, n_mels=128)
# Configuration 1 (tiny, CPU plumbing): 2+2 layers of width 256, 4 heads, FFN 1024,
# depthwise kernel 31, vocabulary 1024; 8x subsampling as in the reference.
TINY_DIMS = dict(enc_d=256, enc_ff=1024, enc_h=4, enc_dk=64, enc_n=2, enc_ck=31, sub_ch=64,
                 dec_d=256, dec_ff=1024, dec_h=4, dec_dk=64, dec_n=2,
                 vocab=1024, max_seq=1024, n_mels=128)

# ---- field order of the weight-table structs (backends/model_types.h:52-77) --

ELAYER_FIELDS = [
    "ff1_lnw", "ff1_lnb", "ff1_w1", "ff1_b1", "ff1_w2", "ff1_b2",
    "sa_lnw", "sa_lnb", "sa_qw", "sa_qb", "sa_kw", "sa_kb",
    "sa_vw", "sa_vb", "sa_pw", "sa_ow", "sa_ob", "sa_pbu", "sa_pbv",
    "cv_lnw", "cv_lnb", "cv_pw1w", "cv_pw1b", "cv_dww", "cv_dwb",
    "cv_bnw", "cv_bnb", "cv_bnmean", "cv_bnvar", "cv_pw2w", "cv_pw2b",
    "ff2_lnw", "ff2_lnb", "ff2_w1", "ff2_b1", "ff2_w2", "ff2_b2",
    "out_lnw", "out_lnb",
]
DLAYER_FIELDS = [
    "sa_lnw", "sa_lnb", "sa_qw", "sa_qb", "sa_kw", "sa_kb", "sa_vw", "sa_vb", "sa_ow", "sa_ob",
    "ca_lnw", "ca_lnb", "ca_qw", "ca_qb", "ca_kw", "ca_kb", "ca_vw", "ca_vb", "ca_ow", "ca_ob",
    "ffn_lnw", "ffn_lnb", "ffn_w1", "ffn_b1", "ffn_w2", "ffn_b2",
]
HEAD_FIELDS = ["s0w", "s0b", "s2w", "s2b", "s3w", "s3b", "s5w", "s5b", "s6w", "s6b", "sow", "sob"]
MID_FIELDS = ["prw", "prb", "etw", "epw", "elnw", "elnb"]
TAIL_FIELDS = ["dlnw", "dlnb", "hdb"]

# Hugging Face tensor names (model.h:160-224 / convert.py:58-154).
_ENC_NAMES = {
    "ff1_lnw": "norm_feed_forward1.weight", "ff1_lnb": "norm_feed_forward1.bias",
    "ff1_w1": "feed_forward1.linear1.weight", "ff1_b1": "feed_forward1.linear1.bias",
    "ff1_w2": "feed_forward1.linear2.weight", "ff1_b2": "feed_forward1.linear2.bias",
    "sa_lnw": "norm_self_att.weight", "sa_lnb": "norm_self_att.bias",
    "sa_qw": "self_attn.linear_q.weight", "sa_qb": "self_attn.linear_q.bias",
    "sa_kw": "self_attn.linear_k.weight", "sa_kb": "self_attn.linear_k.bias",
    "sa_vw": "self_attn.linear_v.weight", "sa_vb": "self_attn.linear_v.bias",
    "sa_pw": "self_attn.linear_pos.weight",
    "sa_ow": "self_attn.linear_out.weight", "sa_ob": "self_attn.linear_out.bias",
    "sa_pbu": "self_attn.pos_bias_u", "sa_pbv": "self_attn.pos_bias_v",
    "cv_lnw": "norm_conv.weight", "cv_lnb": "norm_conv.bias",
    "cv_pw1w": "conv.pointwise_conv1.weight", "cv_pw1b": "conv.pointwise_conv1.bias",
    "cv_dww": "conv.depthwise_conv.weight", "cv_dwb": "conv.depthwise_conv.bias",
    "cv_bnw": "conv.batch_norm.weight", "cv_bnb": "conv.batch_norm.bias",
    "cv_bnmean": "conv.batch_norm.running_mean", "cv_bnvar": "conv.batch_norm.running_var",
    "cv_pw2w": "conv.pointwise_conv2.weight", "cv_pw2b": "conv.pointwise_conv2.bias",
    "ff2_lnw": "norm_feed_forward2.weight", "ff2_lnb": "norm_feed_forward2.bias",
    "ff2_w1": "feed_forward2.linear1.weight", "ff2_b1": "feed_forward2.linear1.bias",
    "ff2_w2": "feed_forward2.linear2.weight", "ff2_b2": "feed_forward2.linear2.bias",
    "out_lnw": "norm_out.weight", "out_lnb": "norm_out.bias",
}
_DEC_NAMES = {
    "sa_lnw": "layer_norm_1.weight", "sa_lnb": "layer_norm_1.bias",
    "sa_qw": "first_sub_layer.query_net.weight", "sa_qb": "first_sub_layer.query_net.bias",
    "sa_kw": "first_sub_layer.key_net.weight", "sa_kb": "first_sub_layer.key_net.bias",
    "sa_vw": "first_sub_layer.value_net.weight", "sa_vb": "first_sub_layer.value_net.bias",
    "sa_ow": "first_sub_layer.out_projection.weight", "sa_ob": "first_sub_layer.out_projection.bias",
    "ca_lnw": "layer_norm_2.weight", "ca_lnb": "layer_norm_2.bias",
    "ca_qw": "second_sub_layer.query_net.weight", "ca_qb": "second_sub_layer.query_net.bias",
    "ca_kw": "second_sub_layer.key_net.weight", "ca_kb": "second_sub_layer.key_net.bias",
    "ca_vw": "second_sub_layer.value_net.weight", "ca_vb": "second_sub_layer.value_net.bias",
    "ca_ow": "second_sub_layer.out_projection.weight", "ca_ob": "second_sub_layer.out_projection.bias",
    "ffn_lnw": "layer_norm_3.weight", "ffn_lnb": "layer_norm_3.bias",
    "ffn_w1": "third_sub_layer.dense_in.weight", "ffn_b1": "third_sub_layer.dense_in.bias",
    "ffn_w2": "third_sub_layer.dense_out.weight", "ffn_b2": "third_sub_layer.dense_out.bias",
}
_FIXED_NAMES = {
    "s0w": "encoder.pre_encode.conv.0.weight", "s0b": "encoder.pre_encode.conv.0.bias",
    "s2w": "encoder.pre_encode.conv.2.weight", "s2b": "encoder.pre_encode.conv.2.bias",
    "s3w": "encoder.pre_encode.conv.3.weight", "s3b": "encoder.pre_encode.conv.3.bias",
    "s5w": "encoder.pre_encode.conv.5.weight", "s5b": "encoder.pre_encode.conv.5.bias",
    "s6w": "encoder.pre_encode.conv.6.weight", "s6b": "encoder.pre_encode.conv.6.bias",
    "sow": "encoder.pre_encode.out.weight", "sob": "encoder.pre_encode.out.bias",
    "prw": "encoder_decoder_proj.weight", "prb": "encoder_decoder_proj.bias",
    "etw": "transf_decoder._embedding.token_embedding.weight",
    "epw": "transf_decoder._embedding.position_embedding.pos_enc",
    "elnw": "transf_decoder._embedding.layer_norm.weight",
    "elnb": "transf_decoder._embedding.layer_norm.bias",
    "dlnw": "transf_decoder._decoder.final_layer_norm.weight",
    "dlnb": "transf_decoder._decoder.final_layer_norm.bias",
    "hdb": "log_softmax.mlp.layer0.bias",
}


def _enc_spec(d, f):
    D, FF, CK = d["enc_d"], d["enc_ff"], d["enc_ck"]
    shapes = {
        "ff1_w1": ((FF, D), "lin"), "ff1_b1": ((FF,), "bias"),
        "ff1_w2": ((D, FF), "lin"), "ff1_b2": ((D,), "bias"),
        "sa_qw": ((D, D), "lin"), "sa_qb": ((D,), "bias"),
        "sa_kw": ((D, D), "lin"), "sa_kb": ((D,), "bias"),
        "sa_vw": ((D, D), "lin"), "sa_vb": ((D,), "bias"),
        "sa_pw": ((D, D), "lin"), "sa_ow": ((D, D), "lin"), "sa_ob": ((D,), "bias"),
        "sa_pbu": ((d["enc_h"], d["enc_dk"]), "bias"), "sa_pbv": ((d["enc_h"], d["enc_dk"]), "bias"),
        "cv_pw1w": ((2 * D, D, 1), "lin"), "cv_pw1b": ((2 * D,), "bias"),
        "cv_dww": ((D, 1, CK), "lin"), "cv_dwb": ((D,), "bias"),
        "cv_bnw": ((D,), "gamma"), "cv_bnb": ((D,), "bias"),
        "cv_bnmean": ((D,), "bnmean"), "cv_bnvar": ((D,), "bnvar"),
        "cv_pw2w": ((D, D, 1), "lin"), "cv_pw2b": ((D,), "bias"),
        "ff2_w1": ((FF, D), "lin"), "ff2_b1": ((FF,), "bias"),
        "ff2_w2": ((D, FF), "lin"), "ff2_b2": ((D,), "bias"),
    }
    if f in shapes:
        return shapes[f]
    return ((D,), "gamma" if f.endswith("lnw") else "bias")


def _dec_spec(d, f):
    D, FF = d["dec_d"], d["dec_ff"]
    if f.endswith("lnw"):
        return ((D,), "gamma")
    if f.endswith("lnb"):
        return ((D,), "bias")
    if f == "ffn_w1":
        return ((FF, D), "lin")
    if f == "ffn_b1":
        return ((FF,), "bias")
    if f == "ffn_w2":
        return ((D, FF), "lin")
    if f.endswith("w"):
        return ((D, D), "lin")
    return ((D,), "bias")


def _fixed_spec(d, f):
    C, D, DD = d["sub_ch"], d["enc_d"], d["dec_d"]
    f3 = ((d["n_mels"] + 1) // 2 + 1) // 2
    f3 = (f3 + 1) // 2
    table = {
        "s0w": ((C, 1, 3, 3), "lin"), "s0b": ((C,), "bias"),
        "s2w": ((C, 1, 3, 3), "lin"), "s2b": ((C,), "bias"),
        "s3w": ((C, C, 1, 1), "lin"), "s3b": ((C,), "bias"),
        "s5w": ((C, 1, 3, 3), "lin"), "s5b": ((C,), "bias"),
        "s6w": ((C, C, 1, 1), "lin"), "s6b": ((C,), "bias"),
        "sow": ((D, C * f3), "lin"), "sob": ((D,), "bias"),
        "prw": ((DD, D), "lin"), "prb": ((DD,), "bias"),
        "etw": ((d["vocab"], DD), "embed"), "epw": ((d["max_seq"], DD), "pos"),
        "elnw": ((DD,), "gamma"), "elnb": ((DD,), "bias"),
        "dlnw": ((DD,), "gamma"), "dlnb": ((DD,), "bias"),
        "hdb": ((d["vocab"],), "bias"),
    }
    return table[f]


def tensor_list(dims: dict, parts=("enc", "dec")):
    """[(hf_name, struct_key, shape, init)] in model order.  struct_key is
    ('fixed', field) / ('enc', layer, field) / ('dec', layer, field)."""
    out = []
    if "enc" in parts:
        for f in HEAD_FIELDS:
            out.append((_FIXED_NAMES[f], ("fixed", f)) + _fixed_spec(dims, f))
        for l in range(dims["enc_n"]):
            for f in ELAYER_FIELDS:
                out.append((f"encoder.layers.{l}.{_ENC_NAMES[f]}", ("enc", l, f)) + _enc_spec(dims, f))
        for f in ("prw", "prb"):
            out.append((_FIXED_NAMES[f], ("fixed", f)) + _fixed_spec(dims, f))
    if "dec" in parts:
        for f in ("etw", "epw", "elnw", "elnb"):
            out.append((_FIXED_NAMES[f], ("fixed", f)) + _fixed_spec(dims, f))
        for l in range(dims["dec_n"]):
            for f in DLAYER_FIELDS:
                out.append((f"transf_decoder._decoder.layers.{l}.{_DEC_NAMES[f]}", ("dec", l, f))
                           + _dec_spec(dims, f))
        for f in TAIL_FIELDS:
            out.append((_FIXED_NAMES[f], ("fixed", f)) + _fixed_spec(dims, f))
    return out


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + r) >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _draw(seed: int, name: str, shape, init: str, dims: dict) -> np.ndarray:
    rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
    n = int(np.prod(shape))
    if init == "lin":
        fan_in = int(np.prod(shape[1:]))
        v = rng.standard_normal(n, dtype=np.float32) * np.float32(1.0 / np.sqrt(fan_in))
    elif init == "bias":
        v = rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
    elif init == "gamma":
        v = np.float32(1.0) + rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
    elif init == "bnmean":
        v = rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)
    elif init == "bnvar":
        v = rng.uniform(0.5, 1.5, n).astype(np.float32)
    elif init == "embed":
        v = rng.standard_normal(n, dtype=np.float32) * np.float32(1.0 / np.sqrt(dims["dec_d"]))
    elif init == "pos":
        v = rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)
    else:
        raise ValueError(init)
    return f32_to_bf16(v)


@dataclass
class WeightBlob:
    """A contiguous bf16 blob plus the placement of every tensor in it."""
    dims: dict
    blob: np.ndarray                      # uint16, 256-byte aligned base
    index: dict = field(default_factory=dict)   # hf_name -> (offset_elems, shape, struct_key)
    parts: tuple = ("enc", "dec")

    @property
    def nbytes(self) -> int:
        return int(self.blob.nbytes)

    def ptr(self) -> int:
        return int(self.blob.ctypes.data)

    def tensor(self, name: str) -> np.ndarray:
        off, shape, _ = self.index[name]
        return self.blob[off:off + int(np.prod(shape))].reshape(shape)

    def field(self, key) -> np.ndarray:
        for name, (off, shape, k) in self.index.items():
            if k == key:
                return self.blob[off:off + int(np.prod(shape))].reshape(shape)
        raise KeyError(key)


def make_blob(dims: dict = FULL_DIMS, seed: int = 0, parts=("enc", "dec")) -> WeightBlob:
    """Generate the random-init blob.  Every tensor starts on a 128-element
    (256-byte) boundary so device copies keep vector alignment."""
    specs = tensor_list(dims, parts)
    offs, total = [], 0
    for _name, _key, shape, _init in specs:
        offs.append(total)
        total += (int(np.prod(shape)) + 127) // 128 * 128
    raw = np.zeros(total + 128, dtype=np.uint16)
    shift = (-raw.ctypes.data // 2) % 128          # align the base to 256 bytes
    blob = raw[shift:shift + total]
    wb = WeightBlob(dims=dims, blob=blob, parts=tuple(parts))

    def fill(i):
        name, key, shape, init = specs[i]
        blob[offs[i]:offs[i] + int(np.prod(shape))] = _draw(seed, name, shape, init, dims)

    # tensors are drawn independently (one generator per name), so threads
    # give the same blob as a serial fill
    with ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as pool:
        list(pool.map(fill, range(len(specs))))
    for (name, key, shape, _init), off in zip(specs, offs):
        wb.index[name] = (off, tuple(shape), key)
    wb._raw = raw  # keep the allocation alive
    return wb


# ---- ctypes mirror of the Weights struct ------------------------------------

def weights_struct_type(enc_n: int, dec_n: int):
    """ctypes type with the layout of `Weights` for the given layer counts
    (all fields are pointers; order as in backends/model_types.h:52-77)."""
    P = ctypes.c_void_p
    EL = type("ELayer", (ctypes.Structure,), {"_fields_": [(f, P) for f in ELAYER_FIELDS]})
    DL = type("DLayer", (ctypes.Structure,), {"_fields_": [(f, P) for f in DLAYER_FIELDS]})
    fields = [(f, P) for f in HEAD_FIELDS] + [("enc", EL * enc_n)] + [(f, P) for f in MID_FIELDS] \
        + [("dec", DL * dec_n)] + [(f, P) for f in TAIL_FIELDS]
    return type("Weights", (ctypes.Structure,), {"_fields_": fields})


def weights_struct(wb: WeightBlob, enc_n: int = 48, dec_n: int = 8):
    """Fill a `Weights` struct with host pointers into wb.blob (NULL for tensors
    the blob does not hold)."""
    WT = weights_struct_type(enc_n, dec_n)
    w = WT()
    base = wb.ptr()
    for name, (off, shape, key) in wb.index.items():
        addr = base + 2 * off
        if key[0] == "fixed":
            setattr(w, key[1], addr)
        elif key[0] == "enc":
            setattr(w.enc[key[1]], key[2], addr)
        else:
            setattr(w.dec[key[1]], key[2], addr)
    return w


def write_safetensors(wb: WeightBlob, path: str) -> None:
    """Write the blob as a safetensors file (bf16, HF names), the format
    model.h's sf_load/sf_get read (model.h:46-81)."""
    header, data_parts, pos = {}, [], 0
    for name, (off, shape, _key) in wb.index.items():
        n = int(np.prod(shape))
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [pos, pos + 2 * n]}
        data_parts.append(wb.blob[off:off + n])
        pos += 2 * n
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(hb)))
        fh.write(hb)
        for part in data_parts:
            fh.write(part.tobytes())
