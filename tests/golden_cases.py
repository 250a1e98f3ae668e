"""Loader for the golden vectors in tests/golden/*.npz (written by tests/golden/make_golden.py
from the compiled reference CPU path)."""
import glob
import json
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def names(pattern="*"):
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, pattern + ".npz")))


def load(name):
    with np.load(os.path.join(GOLDEN_DIR, name + ".npz")) as z:
        d = {k: z[k] for k in z.files}
    if "meta" in d:
        d["meta"] = json.loads(str(d["meta"]))
    return d


def coding_cases():
    """Golden cases holding one push + pop round (everything with a 'pushed' array)."""
    return [n for n in names() if "pushed" in np.load(os.path.join(GOLDEN_DIR, n + ".npz")).files]


def payload_bytes(stream):
    """rans_stream_to_byte_strings of a numpy stream, concatenated (torch_ans/rans.cpp:5-21)."""
    s = np.ascontiguousarray(stream, dtype=np.int32)
    return b"".join(s[b, 1:].tobytes()[: int(s[b, 0])] for b in range(s.shape[0]))
