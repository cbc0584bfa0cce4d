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


def crossfile_case(g, name):
    """Fields of one crossfile.npz case, without the case prefix; the
    segmenter's chunks come back as this library's CodeChunk objects."""
    from sabrecoder_b200.chunks import ChunkType, CodeChunk
    c = {k[len(name) + 1:]: v for k, v in g.items() if k.startswith(name + "_")}
    seg = []
    for i, ch in enumerate(chunks(c, "seg_")):
        seg.append(CodeChunk(ChunkType[ch.chunk_type.name], 0, 0, str(c["seg_texts"][i]), name=ch.name,
                             start_line=ch.start_line, end_line=ch.end_line,
                             signature_start_line=ch.signature_start_line,
                             signature_end_line=ch.signature_end_line))
    c["seg_chunks"] = seg
    c["ref_chunks"] = chunks(c, "ref_")
    c["ref_deps"] = deps(c, "ref_dep_src", "ref_dep_dst")
    return c


def crossfile_builder(c, **extra):
    """A StructureAwareMaskBuilder with the case's parameters and a fixed
    segmenter / analyser standing in for tree-sitter."""
    import torch
    from sabrecoder_b200.sabrecoder_attention import StructureAwareMaskBuilder
    from sabrecoder_b200.spans import HashTokenizer

    class Seg:
        def __init__(self, tokenizer=None):
            pass

        def segment_code(self, code, language=None):
            return list(c["seg_chunks"])

    class Ana:
        def __init__(self, chunks_, code, language=None):
            pass

        def analyze(self):
            return [SimpleNamespace(source_chunk_idx=int(a), target_chunk_idx=int(b))
                    for a, b in zip(c["edge_src"].tolist(), c["edge_dst"].tolist())]

    p = {k[2:]: c[k].item() for k in c if k.startswith("p_")}
    emb = bf16_bits_to_f32(c["emb_bf16"]).to(torch.bfloat16)
    return StructureAwareMaskBuilder(HashTokenizer(128), embedding_weight=emb, segmenter_factory=Seg,
                                     analyzer_factory=Ana, **p, **extra)
