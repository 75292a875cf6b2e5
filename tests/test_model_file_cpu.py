"""The model file this repository writes loads in the reference's own loader.

`weights.write_safetensors` writes the seeded random-init weights as a
safetensors file: bf16 tensors under the Hugging Face names convert.py emits.
The reference's `load_weights` (model.h: sf_load + sf_get by name) then reads
that file, from the library built from the reference sources
(oracle/_ref/libref_decode_tiny.so, configuration 1's dims). The check: it
finds every tensor, and every pointer in the weight table it builds holds
exactly the values of our tensor of that name. The load runs in a child
process, because the reference loader exits on a missing tensor.
"""
import os
import subprocess
import sys
import textwrap

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent("""
    import ctypes, importlib, os, sys
    import numpy as np
    sys.path[:0] = [{repo!r}, os.path.join({repo!r}, "oracle")]
    import pyoracle as po
    W = importlib.import_module("cohere-transcribe_b200.weights")
    wb = W.make_blob(W.TINY_DIMS, seed=2)
    d = {tmp!r}
    os.makedirs(os.path.join(d, "model_files"), exist_ok=True)
    W.write_safetensors(wb, os.path.join(d, "model_files", "model.safetensors"))
    L = po.ref_lib("libref_decode_tiny.so")
    WT = W.weights_struct_type(2, 2)
    out = WT()
    L.refh_load_model_file.argtypes = [ctypes.c_char_p, ctypes.c_void_p]
    assert L.refh_load_model_file(d.encode(), ctypes.addressof(out)) == 0
    n = 0
    for name, (off, shape, key) in wb.index.items():
        if key[0] == "fixed":
            p = getattr(out, key[1])
        elif key[0] == "enc":
            p = getattr(out.enc[key[1]], key[2])
        else:
            p = getattr(out.dec[key[1]], key[2])
        assert p, name
        cnt = int(np.prod(shape))
        got = np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_uint16)), shape=(cnt,))
        assert np.array_equal(got, wb.tensor(name).ravel()), name
        n += 1
    print("tensors", n)
""")


def test_reference_loader_reads_our_model_file(tmp_path):
    if not os.path.exists(os.path.join(REPO, "oracle", "_ref", "libref_decode_tiny.so")):
        pytest.skip("reference decode harness not built (oracle/_ref/ needs the reference tree)")
    r = subprocess.run([sys.executable, "-c", CHILD.format(repo=REPO, tmp=str(tmp_path))], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    n = int(r.stdout.split()[-1])
    assert n > 50
