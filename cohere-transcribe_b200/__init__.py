"""cohere-transcribe B200 backend: host-side Python mirror of the C ABI.

The product is libct_b200.so (CUDA for sm_100a, C ABI declared in include/).
This package holds the build step, ctypes prototypes of that ABI, the seeded
weight generator and the synthetic-input generators used by tests and bench.
The directory name contains a hyphen, so import it with
``importlib.import_module("cohere-transcribe_b200")``.
"""
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
LIB_PATH = os.path.join(PKG_DIR, "libct_b200.so")
INCLUDE_DIR = os.path.join(REPO_DIR, "include")

# The ten prompt tokens of transcribe.c:1320-1330 (pnc on, itn/timestamps/diarize
# off).  The language token id is a fixed synthetic id because the vocabulary
# is synthetic; vocab-1024 models remap TOK_LEADING_SPACE (13764) below VOCAB.
LANG_ID = 62
PROMPT_FULL = [13764, 7, 4, 16, LANG_ID, LANG_ID, 5, 9, 11, 13]
PROMPT_TINY = [13764 % 1024, 7, 4, 16, LANG_ID, LANG_ID, 5, 9, 11, 13]
TOK_EOS = 3


def prompt_tokens(lang_id: int = LANG_ID, pnc: bool = True, itn: bool = False, timestamps: bool = False,
                  diarize: bool = False, leading_space: int = 13764) -> list:
    """The ten prompt tokens of transcribe.c:1320-1330 for one utterance's
    options (token ids of model.h:24-36)."""
    return [leading_space, 7, 4, 16, lang_id, lang_id, 5 if pnc else 6, 8 if itn else 9,
            10 if timestamps else 11, 12 if diarize else 13]


def t_enc_of(t_mel: int) -> int:
    """Encoder frames after 8x subsampling (transcribe.c:268-271)."""
    t1 = (t_mel + 1) // 2
    t2 = (t1 + 1) // 2
    return (t2 + 1) // 2


def t_mel_of_seconds(sec: float) -> int:
    """Log-mel frames for `sec` seconds at 16 kHz, hop 160 (transcribe.c:268)."""
    return 1 + int(round(sec * 16000)) // 160
