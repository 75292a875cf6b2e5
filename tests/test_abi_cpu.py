"""CPU checks of the drop-in boundary (no GPU calls).

* libct_b200.so loads without a GPU and exports every function declared in
  include/*.h (the 40 backend_* symbols of the reference's backends/backend.h).
* The weight-table structs of include/ct_model_types.h have exactly the field
  offsets of the reference's backends/model_types.h (tests/golden/struct_offsets_ref.txt).
* With the reference source tree present, its own transcribe.c and
  tests/test_kernels.c link against the library (the drop-in at link level).
"""
import ctypes
import importlib
import os
import re
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for fn in os.listdir(os.path.join(REPO, "include")):
        if fn.endswith(".h"):
            txt = open(os.path.join(REPO, "include", fn)).read()
            txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
            names |= set(re.findall(r"^\s*(?:[\w\s\*]+?)\b((?:backend|ct|b200)_\w+)\s*\(", txt, flags=re.M))
    return names


def test_library_exports_every_declared_symbol(ctb):
    abi = __import__("importlib").import_module("cohere-transcribe_b200.abi")
    lib = abi.load()
    declared = _declared()
    assert {n for n in declared if n.startswith("backend_")} == set(abi.BACKEND_SYMBOLS)
    assert len(abi.BACKEND_SYMBOLS) == 40
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing


def test_weight_struct_layout_matches_reference(tmp_path):
    exe = tmp_path / "offs"
    hdr = os.path.join(REPO, "include", "ct_model_types.h")
    subprocess.run(["gcc", "-O0", f'-DMODEL_TYPES_HEADER="{hdr}"', "-o", str(exe),
                    os.path.join(REPO, "tests", "golden", "struct_offsets.c")], check=True)
    mine = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    ref = open(os.path.join(REPO, "tests", "golden", "struct_offsets_ref.txt")).read()
    assert mine == ref


def test_ctypes_weights_struct_matches_c_layout(wmod):
    WT = wmod.weights_struct_type(48, 8)
    ref = dict(line.split() for line in open(os.path.join(REPO, "tests", "golden", "struct_offsets_ref.txt")))
    assert ctypes.sizeof(WT) == int(ref["sizeof.Weights"])
    for f in ("etw", "epw", "hdb", "dlnw", "prw"):
        assert getattr(WT, f).offset == int(ref[f"Weights.{f}"])
    assert WT.dec.offset == int(ref["Weights.dec"])


REFERENCE_DIR = importlib.import_module("__graft_entry__").REFERENCE_DIR   # where build() finds the reference


@pytest.mark.skipif(not (REFERENCE_DIR and os.path.exists(os.path.join(REFERENCE_DIR, "transcribe.c"))),
                    reason="needs the reference source tree (set CT_REFERENCE_DIR)")
def test_reference_programs_link_against_the_library(tmp_path):
    """The reference's own host programs -- transcribe.c (with model.h) and
    tests/test_kernels.c, compiled as its build uses them with -DBACKEND_CUDA --
    link against libct_b200.so in place of the CUDA backend object, with every
    backend_* symbol they call resolved by this library.  transcribe.c's
    generated vocabulary header comes from the tokenizer, which is absent here,
    so an empty one stands in (it only feeds detokenisation)."""
    lib_dir = os.path.join(REPO, "cohere-transcribe_b200")
    gen = tmp_path / "gen"
    gen.mkdir()
    (gen / "vocab_txt.h").write_text("unsigned char vocab_txt[] = {0};\nunsigned int vocab_txt_len = 1;\n")
    for src, extra in (("transcribe.c", [f"-I{gen}", "-lpthread"]), (os.path.join("tests", "test_kernels.c"), [])):
        exe = tmp_path / os.path.basename(src).replace(".c", "")
        subprocess.run(["gcc", "-O1", "-DBACKEND_CUDA", f"-I{REFERENCE_DIR}", "-w", "-o", str(exe),
                        os.path.join(REFERENCE_DIR, src), f"-L{lib_dir}", "-lct_b200", f"-Wl,-rpath,{lib_dir}"]
                       + extra + ["-lm"], check=True)
        undefined = subprocess.run(["nm", "-u", str(exe)], capture_output=True, text=True, check=True).stdout
        called = {ln.split()[-1] for ln in undefined.splitlines() if "backend_" in ln}
        assert called, src
        lib = ctypes.CDLL(os.path.join(lib_dir, "libct_b200.so"))
        assert all(hasattr(lib, name) for name in called), src
