"""Helpers to read the committed golden fixtures (tests/golden/*.npz)."""

import glob
import os
from types import SimpleNamespace

import numpy as np

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TYPE_NAMES = {0: "IMPORT", 1: "FUNCTION", 2: "CLASS", 3: "METHOD", 4: "MODULE_CODE", 5: "COMMENT",
              6: "DOCSTRING"}


def load(name):
    return dict(np.load(os.path.join(HERE, name), allow_pickle=False))


def mask_cases():
    return sorted(os.path.basename(p) for p in glob.glob(os.path.join(HERE, "mask_*.npz")))


def chunks(g, prefix=""):
    out = []
    for i in range(g[prefix + "chunk_type"].shape[0]):
        s0 = int(g[prefix + "chunk_sig_start"][i])
        s1 = int(g[prefix + "chunk_sig_end"][i])
        out.append(SimpleNamespace(
            chunk_type=SimpleNamespace(name=TYPE_NAMES[int(g[prefix + "chunk_type"][i])]),
            chunk_type_code=int(g[prefix + "chunk_type"][i]),
            start_line=int(g[prefix + "chunk_start_line"][i]),
            end_line=int(g[prefix + "chunk_end_line"][i]),
            signature_start_line=s0 or None, signature_end_line=s1 or None,
            name=str(g[prefix + "chunk_name"][i])))
    return out


def deps(g, src="dep_src", dst="dep_dst"):
    d = {}
    for s, t in zip(g[src].tolist(), g[dst].tolist()):
        d.setdefault(int(s), set()).add(int(t))
    return d


def params(g):
    return {k[2:]: int(g[k]) for k in g if k.startswith("p_")}


def tokenizer(g):
    from sabrecoder_b200.spans import LineTokenizer, WordTokenizer
    return WordTokenizer() if str(g["tokenizer"]) == "word-tokenizer" else LineTokenizer()


def bf16_bits_to_f32(a):
    import torch
    return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16).float()
