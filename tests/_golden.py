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


def bf16_bits_to_np(a):
    """uint16 bf16 bit patterns -> float32 numpy array."""
    return (a.astype(np.uint32) << 16).view(np.float32)


SIM_PARAM_KEYS = ("chunk_similarity_top_percent", "chunk_similarity_max_neighbors",
                  "chunk_similarity_max_tokens_per_chunk")


def sim_case(g, name):
    """(texts, embedding fp32, params, src, tgt, edges) of a similarity.npz case."""
    texts = [str(t) for t in g[f"{name}_texts"]]
    emb = bf16_bits_to_np(g[f"{name}_emb_bf16"])
    p = {k: g[f"{name}_p_{k}"].item() for k in SIM_PARAM_KEYS}
    sub = bool(g[f"{name}_has_subsets"])
    src = g[f"{name}_src"].tolist() if sub else None
    tgt = g[f"{name}_tgt"].tolist() if sub else None
    edges = deps(g, f"{name}_edge_src", f"{name}_edge_dst")
    return texts, emb, p, src, tgt, edges


def token_cases():
    return sorted(os.path.basename(p) for p in glob.glob(os.path.join(HERE, "token_*.npz")))


def token_visible(g):
    """The reference's token-level visibility restricted to key <= query."""
    L = int(g["seq_len"])
    vis = np.unpackbits(g["visible_bits"], axis=-1)[:, :L].astype(bool)
    return vis & np.tril(np.ones((L, L), dtype=bool))
