"""Record golden vectors from the reference implementation.

Runs only where the reference checkout is present; the GPU machines and the
test suite use the committed ``.npz`` files instead. Regenerate with::

    python tests/golden/gen_golden.py --reference <checkout of SabreCoder>

(or set ``SABRECODER_REF`` to the checkout).

What is recorded (all from the reference's own code, unmodified):

* ``mask_*.npz`` -- ``StructureAwareMaskBuilder._build_block_mask_from_chunks``
  (methods/sabrecoder/sabrecoder_attention_triton.py:1455-1604) on seeded
  synthetic chunk sets, plus the token-level inputs the reference derives
  (``_map_tokens_to_chunks`` :807-858, signature/special lines mapped to
  tokens :1557-1572), and ``compute_block_indices_from_mask`` (:1837-1859)
  both raw and canonicalised (rows sorted).
* ``mask_pyspecial.npz`` -- the Python special-line rules (:697-752) on a
  synthetic Python-like file with a multi-token-per-line tokenizer.
* ``builder_full.npz`` -- ``build_block_indices`` (:1606-1819) end to end with
  the segmenter and reference analyser replaced by fixed chunk/edge lists
  (tree-sitter is not installed), covering ``_append_uncovered_line_chunks``.
* ``attn_*.npz`` -- ``_fwd_kernel_sabrecoder`` (:28-116) run by Triton's
  interpreter in fp32 on bf16-representable inputs.
* ``sparsity_utils.json`` -- utils/sparsity_utils.py values.
* ``token_*.npz`` -- ``_build_mask_from_chunks`` (:1171-1266, the token-level
  mask of ``use_token_level_sparsity=True``) on seeded chunk sets, stored as
  packed visibility bits, and ``_fwd_kernel_sabrecoder_token_sparse``
  (:119-215) run by Triton's interpreter in fp32 with that mask.
* ``similarity.npz`` -- ``_similarity_edges`` (:581-682, with
  ``_get_or_build_similarity_vectors`` :490-579 and ``_clean_for_similarity``
  :458-472) on seeded chunk texts and a seeded bf16 embedding table, for
  three parameter sets, and ``build_block_indices`` end to end with
  ``use_chunk_similarity=True``.

The tree-sitter modules (pinned tree-sitter==0.20.4,
tree-sitter-languages==1.10.2 in the reference's requirements.txt) are
replaced by empty stand-ins so the module imports; nothing here parses code.
"""

from __future__ import annotations

import json
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"


def _reference_root() -> str:
    """The reference checkout: ``--reference PATH`` or ``$SABRECODER_REF``."""
    for i, a in enumerate(sys.argv[1:], 1):
        if a == "--reference" and i + 1 < len(sys.argv):
            return sys.argv[i + 1]
        if a.startswith("--reference="):
            return a.split("=", 1)[1]
    ref = os.environ.get("SABRECODER_REF")
    if not ref:
        sys.exit("gen_golden.py: give the reference checkout with --reference PATH or SABRECODER_REF")
    return ref


REF = _reference_root()
if not os.path.isdir(os.path.join(REF, "methods", "sabrecoder")):
    sys.exit(f"gen_golden.py: {REF} does not hold methods/sabrecoder")
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

for _name in ("tree_sitter_languages", "tree_sitter"):
    _m = types.ModuleType(_name)
    _m.get_parser = lambda *a, **k: None
    _m.Node = object
    sys.modules[_name] = _m
sys.path.insert(0, os.path.join(REF, "methods", "sabrecoder"))
sys.path.insert(0, REF)
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import sabrecoder_attention_triton as R  # noqa: E402
from semantic_chunker import ChunkType, CodeChunk  # noqa: E402
from utils import sparsity_utils as SU  # noqa: E402

from sabrecoder_b200.spans import (HashTokenizer, LineTokenizer, WordTokenizer, make_spans,  # noqa: E402
                                   spans_to_code)

_TYPE = {"import": ChunkType.IMPORT, "function": ChunkType.FUNCTION, "class": ChunkType.CLASS,
         "statement": ChunkType.MODULE_CODE}
_TYPE_CODE = {ChunkType.IMPORT: 0, ChunkType.FUNCTION: 1, ChunkType.CLASS: 2, ChunkType.METHOD: 3,
              ChunkType.MODULE_CODE: 4, ChunkType.COMMENT: 5, ChunkType.DOCSTRING: 6}


def chunks_from_spanset(ss):
    out = []
    for s in ss.spans:
        sig = s.start + 1 if s.has_signature else None
        out.append(CodeChunk(_TYPE[s.tag], 0, 0, "", name=f"s{s.start}", start_line=s.start + 1,
                             end_line=s.end + 1, signature_start_line=sig, signature_end_line=sig))
    return out


def deps_to_arrays(deps):
    src, dst = [], []
    for s in sorted(deps):
        for t in sorted(deps[s]):
            src.append(int(s))
            dst.append(int(t))
    return np.asarray(src, np.int32), np.asarray(dst, np.int32)


def chunk_arrays(chunks):
    return dict(
        chunk_type=np.asarray([_TYPE_CODE[c.chunk_type] for c in chunks], np.int32),
        chunk_start_line=np.asarray([c.start_line for c in chunks], np.int32),
        chunk_end_line=np.asarray([c.end_line for c in chunks], np.int32),
        chunk_sig_start=np.asarray([c.signature_start_line or 0 for c in chunks], np.int32),
        chunk_sig_end=np.asarray([c.signature_end_line or 0 for c in chunks], np.int32),
        chunk_name=np.asarray([c.name or "" for c in chunks]),
    )


def record_mask(name, *, code, seq_len, chunks, deps, imports, language, tok, params):
    mb = R.StructureAwareMaskBuilder(tok, **params)
    bm = mb._build_block_mask_from_chunks(code=code, seq_len=seq_len, chunks=chunks,
                                          chunk_deps=deps, import_chunks=imports, language=language)
    t2c = np.asarray(mb._map_tokens_to_chunks(code, chunks, seq_len), np.int32)
    vis = set()
    for ch in chunks:
        if ch.chunk_type in (ChunkType.FUNCTION, ChunkType.CLASS, ChunkType.METHOD):
            if ch.signature_start_line and ch.signature_end_line:
                vis.update(range(ch.signature_start_line, ch.signature_end_line + 1))
    sp = mb._identify_special_lines(code, chunks, language=language)
    for key in ("global_vars", "type_aliases", "class_attrs", "return_stmts"):
        vis |= sp[key]
    gtm = mb._map_lines_to_tokens(code, vis, seq_len).numpy().astype(np.uint8)
    raw_idx, cnt = R.compute_block_indices_from_mask(bm.unsqueeze(0))
    nb = bm.shape[0]
    canon = np.full(raw_idx.shape, -1, np.int32)
    for r in range(nb):
        c = int(cnt[0, r])
        canon[0, r, :c] = np.sort(raw_idx[0, r, :c].numpy())
    dsrc, ddst = deps_to_arrays(deps)
    np.savez_compressed(
        os.path.join(HERE, f"mask_{name}.npz"),
        code=np.asarray(code), seq_len=seq_len, language=np.asarray(language or ""),
        tokenizer=np.asarray(tok.name_or_path), **{f"p_{k}": v for k, v in params.items()},
        **chunk_arrays(chunks), dep_src=dsrc, dep_dst=ddst,
        import_chunks=np.asarray(sorted(imports), np.int32),
        token_to_chunk=t2c, global_token_mask=gtm, block_mask=bm.numpy().astype(np.uint8),
        raw_indices=raw_idx.numpy(), block_counts=cnt.numpy(), indices_sorted=canon)
    print(f"mask_{name}: L={seq_len} nb={nb} max_active={raw_idx.shape[-1]} "
          f"density={float(bm.sum()) / (nb * (nb + 1) / 2):.3f}")


def synthetic_python_file(seed, n_units=40):
    """A Python-like file from fixed templates, and its chunk list."""
    rng = np.random.default_rng(seed)
    lines, chunks = [], []

    def add(kind, body, name="", sig=True):
        s = len(lines) + 1
        lines.extend(body)
        e = len(lines)
        sl = s if sig else None
        chunks.append(CodeChunk(kind, 0, 0, "\n".join(body), name=name, start_line=s, end_line=e,
                                signature_start_line=sl, signature_end_line=sl))

    add(ChunkType.IMPORT, ["import os", "from typing import List"], sig=False)
    for u in range(n_units):
        r = rng.random()
        if r < 0.2:
            lines.append(f"CONST_{u} = {u}")
            lines.append(f"Alias{u} = List[int]")
            lines.append("# note about constants")
            lines.append("")
        elif r < 0.5:
            s = len(lines) + 1
            body = [f"class K{u}:", "    def __init__(self, a):", "        self.a = a",
                    "        self.b = a == 1", "        return None", f"    def m{u}(self):",
                    "        return self.a"]
            lines.extend(body)
            chunks.append(CodeChunk(ChunkType.CLASS, 0, 0, "", name=f"K{u}", start_line=s,
                                    end_line=s + 6, signature_start_line=s, signature_end_line=s))
            chunks.append(CodeChunk(ChunkType.METHOD, 0, 0, "", name="__init__", start_line=s + 1,
                                    end_line=s + 4, signature_start_line=s + 1, signature_end_line=s + 1))
            chunks.append(CodeChunk(ChunkType.METHOD, 0, 0, "", name=f"m{u}", start_line=s + 5,
                                    end_line=s + 6, signature_start_line=s + 5, signature_end_line=s + 5))
        else:
            n = int(rng.integers(2, 9))
            body = [f"def f{u}(x, y):"] + ["    z = x + y" for _ in range(n)] + ["    if x >= y:",
                                                                               "        return z", "    return x"]
            add(ChunkType.FUNCTION, body, name=f"f{u}")
    return "\n".join(lines), chunks


class _Ref:
    def __init__(self, s, t):
        self.source_chunk_idx, self.target_chunk_idx = s, t


def record_builder_full():
    """build_block_indices end to end with a fixed segmenter/analyser."""
    L = 1500
    ss = make_spans(L, seed=77, max_len=120, p_function=0.4)
    chunks = chunks_from_spanset(ss)
    # Leave every 5th statement chunk out so _append_uncovered_line_chunks fills it.
    seg_chunks = [c for i, c in enumerate(chunks) if not (c.chunk_type == ChunkType.MODULE_CODE and i % 5 == 0)]
    edges = []
    fun = [i for i, c in enumerate(seg_chunks) if c.chunk_type == ChunkType.FUNCTION]
    for a, b in zip(fun[1::2], fun[::2]):
        edges.append((a, b))

    class Seg:
        def __init__(self, tokenizer=None):
            pass

        def segment_code(self, code, language=None):
            return list(seg_chunks)

    class Ana:
        def __init__(self, chunks, code, language=None):
            pass

        def analyze(self):
            return [_Ref(a, b) for a, b in edges]

    R.TreeSitterSegmenter, R.CrossReferenceAnalyzer = Seg, Ana
    code = spans_to_code(ss)
    params = dict(window_size=128, num_prefix_tokens=64, num_suffix_tokens=100, block_size=64,
                  global_last_k_chunks=2, max_chunk_tokens=128)
    mb = R.StructureAwareMaskBuilder(LineTokenizer(), **params)
    bi, bc, bm = mb.build_block_indices(code, L, torch.device("cpu"), batch_size=2)
    filled = mb._append_uncovered_line_chunks(code, seg_chunks)
    nb = bm.shape[0]
    canon = np.full(bi.shape, -1, np.int32)
    for b in range(bi.shape[0]):
        for r in range(nb):
            c = int(bc[b, r])
            canon[b, r, :c] = np.sort(bi[b, r, :c].numpy())
    np.savez_compressed(
        os.path.join(HERE, "builder_full.npz"), code=np.asarray(code), seq_len=L,
        **{f"p_{k}": v for k, v in params.items()}, **chunk_arrays(seg_chunks),
        **{f"filled_{k}": v for k, v in chunk_arrays(filled).items()},
        edge_src=np.asarray([a for a, _ in edges], np.int32),
        edge_dst=np.asarray([b for _, b in edges], np.int32),
        block_mask=bm.numpy().astype(np.uint8), block_counts=bc.numpy(), indices_sorted=canon,
        raw_indices=bi.numpy())
    print(f"builder_full: nb={nb} chunks {len(seg_chunks)} -> {len(filled)} edges={len(edges)}")


def similarity_texts(seed, n_chunks=60):
    """Chunk texts with shared and private identifiers, commented lines (the
    cleaning rule), a blank chunk and a comment-marker-only chunk."""
    rng = np.random.default_rng(seed)
    shared = [f"w{i}" for i in range(40)]
    texts = []
    for c in range(n_chunks):
        if c == 7:
            texts.append("   \n  ")
            continue
        if c == 11:
            texts.append("# \n// ")
            continue
        lines = []
        for _ in range(int(rng.integers(1, 6))):
            words = [shared[int(rng.integers(0, len(shared)))] for _ in range(int(rng.integers(1, 7)))]
            words.append(f"p{c}_{int(rng.integers(0, 3))}")
            pre = ["", "", "# ", "// ", "#"][int(rng.integers(0, 5))]
            lines.append(pre + " ".join(words))
        texts.append("\n".join(lines))
    return texts


def record_similarity():
    """_similarity_edges for three parameter sets, and build_block_indices with
    use_chunk_similarity=True end to end."""
    tok = HashTokenizer(vocab=128)
    out = {}

    def bf16_bits(t):
        return t.view(torch.int16).numpy().view(np.uint16)

    cases = [("a", 0, 200, dict(chunk_similarity_top_percent=0.1, chunk_similarity_max_neighbors=8,
                                 chunk_similarity_max_tokens_per_chunk=256), None, None),
             ("b", 1, 256, dict(chunk_similarity_top_percent=25, chunk_similarity_max_neighbors=3,
                                 chunk_similarity_max_tokens_per_chunk=5), None, None),
             ("c", 2, 128, dict(chunk_similarity_top_percent=0.5, chunk_similarity_max_neighbors=4,
                                 chunk_similarity_max_tokens_per_chunk=64), list(range(10, 60)), list(range(0, 10)))]
    for name, seed, dim, params, src, tgt in cases:
        texts = similarity_texts(100 + seed)
        g = torch.Generator().manual_seed(200 + seed)
        emb = torch.randn(128, dim, generator=g).to(torch.bfloat16)
        chunks = [CodeChunk(ChunkType.MODULE_CODE, 0, 0, t, name=f"c{i}", start_line=i + 1, end_line=i + 1)
                  for i, t in enumerate(texts)]
        mb = R.StructureAwareMaskBuilder(tok, use_chunk_similarity=True, embedding_weight=emb, **params)
        edges = mb._similarity_edges(chunks, f"code-{name}", src_indices=src, tgt_indices=tgt)
        esrc, edst = deps_to_arrays(edges)
        out.update({f"{name}_texts": np.asarray(texts), f"{name}_emb_bf16": bf16_bits(emb),
                    f"{name}_src": np.asarray(src if src is not None else [], np.int32),
                    f"{name}_tgt": np.asarray(tgt if tgt is not None else [], np.int32),
                    f"{name}_has_subsets": np.asarray(src is not None),
                    f"{name}_edge_src": esrc, f"{name}_edge_dst": edst,
                    **{f"{name}_p_{k}": np.asarray(v) for k, v in params.items()}})
        print(f"similarity {name}: dim={dim} chunks={len(texts)} edges={len(esrc)}")

    # end to end: fixed segmenter/analyser, similarity edges merged into R2
    L = 900
    texts = similarity_texts(7, n_chunks=45)
    lines, chunks = [], []
    for i, t in enumerate(texts):
        s0 = len(lines) + 1
        body = t.split("\n")
        lines.extend(body)
        chunks.append(CodeChunk(ChunkType.FUNCTION if i % 4 == 0 else ChunkType.MODULE_CODE, 0, 0, t,
                                name=f"c{i}", start_line=s0, end_line=len(lines),
                                signature_start_line=s0 if i % 4 == 0 else None,
                                signature_end_line=s0 if i % 4 == 0 else None))
    code = "\n".join(lines)

    class Seg:
        def __init__(self, tokenizer=None):
            pass

        def segment_code(self, code, language=None):
            return list(chunks)

    class Ana:
        def __init__(self, chunks, code, language=None):
            pass

        def analyze(self):
            return [_Ref(4, 0)]

    R.TreeSitterSegmenter, R.CrossReferenceAnalyzer = Seg, Ana
    g = torch.Generator().manual_seed(300)
    emb = torch.randn(128, 256, generator=g).to(torch.bfloat16)
    params = dict(window_size=64, num_prefix_tokens=16, num_suffix_tokens=32, block_size=16,
                  global_last_k_chunks=1, max_chunk_tokens=0)
    sim = dict(chunk_similarity_top_percent=0.1, chunk_similarity_max_neighbors=8,
               chunk_similarity_max_tokens_per_chunk=256)
    mb = R.StructureAwareMaskBuilder(tok, use_chunk_similarity=True, embedding_weight=emb, **params, **sim)
    bi, bc, bm = mb.build_block_indices(code, L, torch.device("cpu"))
    nb = bm.shape[0]
    canon = np.full(bi.shape, -1, np.int32)
    for r in range(nb):
        c = int(bc[0, r])
        canon[0, r, :c] = np.sort(bi[0, r, :c].numpy())
    out.update({"e2e_code": np.asarray(code), "e2e_seq_len": L, "e2e_emb_bf16": bf16_bits(emb),
                **{f"e2e_p_{k}": np.asarray(v) for k, v in {**params, **sim}.items()},
                **{f"e2e_{k}": v for k, v in chunk_arrays(chunks).items()},
                "e2e_texts": np.asarray(texts), "e2e_block_mask": bm.numpy().astype(np.uint8),
                "e2e_block_counts": bc.numpy(), "e2e_indices_sorted": canon})
    np.savez_compressed(os.path.join(HERE, "similarity.npz"), **out)
    print(f"similarity e2e: nb={nb} density={float(bm.sum()) / (nb * (nb + 1) / 2):.3f}")


def record_token_level(name, L, seed, over, tok, language=None, attn_heads=0):
    """The reference's token-level mask (and, for small cases, its token-level
    kernel) on a seeded chunk set."""
    base = dict(window_size=64, num_prefix_tokens=16, num_suffix_tokens=32, block_size=64,
                global_last_k_chunks=2, max_chunk_tokens=0)
    params = dict(base, **over)
    if language == "python":
        code, chunks = synthetic_python_file(seed)
        deps = {}
        imports = {i for i, c in enumerate(chunks) if c.chunk_type == ChunkType.IMPORT}
    else:
        ss = make_spans(L, seed, min_len=8, max_len=48, p_function=0.4)
        code = spans_to_code(ss)
        chunks = chunks_from_spanset(ss)
        deps = {int(k): set(int(x) for x in v) for k, v in ss.deps.items()}
        deps.setdefault(0, set()).add(len(chunks) + 3)  # out of range: skipped
        imports = set(ss.import_chunks)
    mb = R.StructureAwareMaskBuilder(tok, **params)
    mask = mb._build_mask_from_chunks(code, L, torch.device("cpu"), torch.float32, chunks, deps, imports,
                                      language=language)
    vis = (mask == 0).numpy()
    dsrc, ddst = deps_to_arrays(deps)
    out = dict(code=np.asarray(code), seq_len=L, language=np.asarray(language or ""),
               tokenizer=np.asarray(tok.name_or_path), **{f"p_{k}": v for k, v in params.items()},
               **chunk_arrays(chunks), dep_src=dsrc, dep_dst=ddst,
               import_chunks=np.asarray(sorted(imports), np.int32), visible_bits=np.packbits(vis, axis=-1))
    if attn_heads:
        g = torch.Generator().manual_seed(seed + 50)
        q, k, v = [torch.randn(1, attn_heads, L, 128, generator=g).to(torch.bfloat16).float() for _ in range(3)]
        bm = R.compute_block_mask_from_token_mask(mask, 64, 64).unsqueeze(0).contiguous()
        bi, bc = R.compute_block_indices_from_mask(bm)
        o = torch.empty_like(q)
        nb = (L + 63) // 64
        R._fwd_kernel_sabrecoder_token_sparse[(nb, attn_heads)](
            q, k, v, o, bi, bc, mask, *q.stride(), *k.stride(), *v.stride(), *o.stride(), *bi.stride(),
            *bc.stride(), *mask.stride(), 1, attn_heads, L, max_active_blocks=bi.shape[2], BLOCK_M=64,
            BLOCK_N=64, BLOCK_DMODEL=128)

        def bits(x):
            return x.to(torch.bfloat16).view(torch.int16).numpy()

        out.update(q_bf16=bits(q), k_bf16=bits(k), v_bf16=bits(v), out=o.numpy(), block_mask=bm[0].numpy())
    np.savez_compressed(os.path.join(HERE, f"token_{name}.npz"), **out)
    print(f"token_{name}: L={L} visible={vis.mean():.3f} chunks={len(chunks)}")


def record_attention(name, B, H, L, D, block, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v = [torch.randn(B, H, L, D, generator=g).to(torch.bfloat16).float() for _ in range(3)]
    nb = (L + block - 1) // block
    bm = (torch.rand(B, nb, nb, generator=g) < 0.5).int()
    bm = bm | torch.eye(nb, dtype=torch.int32)
    bm = torch.tril(bm)
    bi, bc = R.compute_block_indices_from_mask(bm)
    out = torch.empty_like(q)
    R._fwd_kernel_sabrecoder[(nb, B * H)](
        q, k, v, out, bi, bc, *q.stride(), *k.stride(), *v.stride(), *out.stride(), *bi.stride(),
        *bc.stride(), B, H, L, max_active_blocks=bi.shape[2], BLOCK_M=block, BLOCK_N=block,
        BLOCK_DMODEL=D)

    def bits(x):
        return x.to(torch.bfloat16).view(torch.int16).numpy()

    np.savez_compressed(os.path.join(HERE, f"attn_{name}.npz"), q_bf16=bits(q), k_bf16=bits(k),
                        v_bf16=bits(v), block_indices=bi.numpy(), block_counts=bc.numpy(),
                        block_size=block, out=out.numpy())
    print(f"attn_{name}: B={B} H={H} L={L} block={block} max_active={bi.shape[2]}")


def record_sparsity_utils():
    vals = {
        "causal_total_blocks": [[m, n, SU.causal_total_blocks(m, n)] for m, n in
                                [(0, 0), (1, 1), (5, 5), (7, 3), (3, 7), (256, 256), (192, 100)]],
        "ceil_div": [[a, b, SU.ceil_div(a, b)] for a, b in [(0, 64), (1, 64), (64, 64), (65, 64), (16383, 64)]],
    }
    km = [0] * 1000
    for i in (3, 70, 71, 500, 999):
        km[i] = 1
    vals["window_plus_keys"] = [
        [L, w, bs, list(SU.causal_active_blocks_window_plus_keys(L, w, key_token_mask=km[:L] if L == 1000 else None,
                                                                   block_size=bs))]
        for L, w, bs in [(1000, 0, 64), (1000, 64, 64), (1000, 192, 64), (1000, 100, 128), (4096, 192, 64),
                         (0, 64, 64)]]
    vals["attend_ratio_from_cap"] = [[L, c, SU.causal_attend_ratio_from_cap(L, c)] for L, c in
                                     [(100, 10), (4096, 300.5), (0, 1), (10, 100)]]
    with open(os.path.join(HERE, "sparsity_utils.json"), "w") as f:
        json.dump(vals, f, indent=1)
    print("sparsity_utils.json")


def crossfile_prompt(seed, n_segs, java=False, lead=()):
    """A seeded cross-file prompt in the evaluator's format: retrieved segments
    as commented lines under "<mark> <path>: <start> - <end>" headers (plus
    look-alike lines that are not headers and blank lines), then the current
    file as chunk texts; returns (crossfile, current, current chunk list)."""
    rng = np.random.default_rng(seed)
    mark = "// " if java else "# "
    shared = [f"w{i}" for i in range(40)]
    cf = list(lead)
    for s in range(n_segs):
        a = int(rng.integers(1, 200))
        cf.append(f"{mark}pkg/m{s}.{'java' if java else 'py'}: {a} - {a + int(rng.integers(3, 30))}" +
                  ("   " if s % 3 == 1 else ""))
        for _ in range(int(rng.integers(2, 9))):
            words = [shared[int(rng.integers(0, len(shared)))] for _ in range(int(rng.integers(1, 6)))]
            cf.append(mark + " ".join(words) + f" s{s}")
        if s % 4 == 2:
            cf.append(f"{mark}note: 3 - x")      # trailing text: not a header
            cf.append(mark.strip() + f"pkg/z.py: 1 - 2")  # no space after the mark: not a header
        if s % 2 == 0:
            cf.append("")
    crossfile = "\n".join(cf) + "\n\n"
    texts = similarity_texts(seed + 1, n_chunks=30)
    lines, chunks = [], []
    for i, t in enumerate(texts):
        s0 = len(lines) + 1
        lines.extend(t.split("\n"))
        kind = ChunkType.IMPORT if i < 2 else (ChunkType.FUNCTION if i % 4 == 0 else ChunkType.MODULE_CODE)
        if i % 6 == 5:
            continue  # left for the gap filler
        sig = s0 if kind == ChunkType.FUNCTION else None
        chunks.append(CodeChunk(kind, 0, 0, t, name=f"c{i}", start_line=s0, end_line=len(lines),
                                signature_start_line=sig, signature_end_line=sig))
    return crossfile, "\n".join(lines), chunks


def record_crossfile():
    """build_block_indices and build_token_level_mask with crossfile_code /
    current_code (reference :1622-1772, :860-1081): the chunks, edges and
    imports the reference assembles (captured from its
    _build_block_mask_from_chunks call) and its block and token masks."""
    tok = HashTokenizer(vocab=128)
    out = {}
    cases = [
        # name, seed, segments, java, lead lines, full attention, similarity, crossfile similarity, block
        ("full", 40, 6, False, (), True, True, True, 16),
        ("seg", 41, 9, False, ("", "  "), False, True, True, 16),
        ("segjava", 42, 7, True, ("// leading w1 w2", ""), False, False, False, 32),
        ("segtok", 43, 5, False, (), False, True, False, 64),
    ]
    for name, seed, nseg, java, lead, full, sim, cfsim, block in cases:
        crossfile, current, seg_chunks = crossfile_prompt(seed, nseg, java, lead)
        code = crossfile + current
        L = len(tok(code)["input_ids"])
        fun = [i for i, c in enumerate(seg_chunks) if c.chunk_type == ChunkType.FUNCTION]
        edges = [(a, b) for a, b in zip(fun[1::2], fun[::2])]

        class Seg:
            def __init__(self, tokenizer=None):
                pass

            def segment_code(self, code, language=None):
                return list(seg_chunks)

        class Ana:
            def __init__(self, chunks, code, language=None):
                pass

            def analyze(self):
                return [_Ref(a, b) for a, b in edges]

        R.TreeSitterSegmenter, R.CrossReferenceAnalyzer = Seg, Ana
        g = torch.Generator().manual_seed(seed + 500)
        emb = torch.randn(128, 128, generator=g).to(torch.bfloat16)
        params = dict(window_size=32, num_prefix_tokens=8, num_suffix_tokens=24, block_size=block,
                      global_last_k_chunks=1, max_chunk_tokens=0)
        simp = dict(use_chunk_similarity=sim, embedding_weight=emb, chunk_similarity_top_percent=0.2,
                    chunk_similarity_max_neighbors=3, chunk_similarity_max_tokens_per_chunk=64,
                    use_crossfile_chunk_similarity=cfsim, crossfile_chunk_similarity_top_percent=0.3)
        mb = R.StructureAwareMaskBuilder(tok, **params, **simp)
        seen = {}
        inner = mb._build_block_mask_from_chunks

        def spy(**kw):
            seen.update(kw)
            return inner(**kw)

        mb._build_block_mask_from_chunks = spy
        bi, bc, bm = mb.build_block_indices(code, L, torch.device("cpu"), crossfile_code=crossfile,
                                            current_code=current, crossfile_full_attention=full)
        nb = bm.shape[0]
        canon = np.full(bi.shape, -1, np.int32)
        for r in range(nb):
            c = int(bc[0, r])
            canon[0, r, :c] = np.sort(bi[0, r, :c].numpy())
        esrc, edst = deps_to_arrays(seen["chunk_deps"])
        rec = {"code": np.asarray(code), "crossfile": np.asarray(crossfile), "current": np.asarray(current),
               "seq_len": L, "full_attention": np.asarray(full), "emb_bf16": emb.view(torch.int16).numpy(),
               **{f"p_{k}": np.asarray(v) for k, v in params.items()},
               **{f"p_{k}": np.asarray(v) for k, v in simp.items() if k != "embedding_weight"},
               **{f"seg_{k}": v for k, v in chunk_arrays(seg_chunks).items()},
               "seg_texts": np.asarray([c.text for c in seg_chunks]),
               "edge_src": np.asarray([a for a, _ in edges], np.int32),
               "edge_dst": np.asarray([b for _, b in edges], np.int32),
               **{f"ref_{k}": v for k, v in chunk_arrays(seen["chunks"]).items()},
               "ref_texts": np.asarray([c.text for c in seen["chunks"]]),
               "ref_dep_src": esrc, "ref_dep_dst": edst,
               "ref_imports": np.asarray(sorted(seen["import_chunks"]), np.int32),
               "block_mask": bm.numpy().astype(np.uint8), "block_counts": bc.numpy(), "indices_sorted": canon}
        if block == 64:
            mask = mb.build_token_level_mask(code, L, torch.device("cpu"), torch.float32, crossfile_code=crossfile,
                                             current_code=current, crossfile_full_attention=full)
            rec["visible_bits"] = np.packbits((mask == 0).numpy(), axis=-1)
        out.update({f"{name}_{k}": v for k, v in rec.items()})
        print(f"crossfile {name}: L={L} nb={nb} chunks={len(seen['chunks'])} edges={len(esrc)} "
              f"density={float(bm.sum()) / (nb * (nb + 1) / 2):.3f}")
    out["cases"] = np.asarray([c[0] for c in cases])
    np.savez_compressed(os.path.join(HERE, "crossfile.npz"), **out)


# --------------------------------------------------------------------------
# Structure analysis (segmenter + cross-reference analyser) for Python.
# tree-sitter is not installed here, so the reference's TreeSitterSegmenter and
# CrossReferenceAnalyzer are driven through a stand-in parser that presents the
# standard ast module's tree with tree-sitter-python's node types and fields
# (function_definition, class_definition, import_statement,
# import_from_statement, call/function, attribute, identifier, ...). The
# fixtures therefore pin the reference's rules (walk, chunk kinds, names, gap
# filling, callee matching) on ast's parse of the source; tree-sitter's own
# parse is the part they cannot pin.
# --------------------------------------------------------------------------
import ast as _ast  # noqa: E402
import re as _re  # noqa: E402


class _TSNode:
    def __init__(self, kind, a, b, pa, pb, children=(), fields=None):
        self.type = kind
        self.start_byte, self.end_byte = a, b
        self.start_point, self.end_point = pa, pb
        self.children = list(children)
        self.named_children = self.children
        self._fields = fields or {}

    def child_by_field_name(self, name):
        return self._fields.get(name)


class _TSTree:
    def __init__(self, root):
        self.root_node = root


class _AstAsTreeSitter:
    """parse(bytes) -> a tree-sitter-shaped tree built from ast."""

    def parse(self, data):
        code = data.decode("utf-8")
        self.data = data
        self.starts = [0] + [m.end() for m in _re.finditer(b"\n", data)]
        mod = _ast.parse(code)
        kids = [self.conv(n) for n in mod.body]
        end = len(data)
        return _TSTree(_TSNode("module", 0, end, (0, 0), self.point(end), kids))

    def point(self, byte):
        row = max(i for i, st in enumerate(self.starts) if st <= byte)
        return (row, byte - self.starts[row])

    def pos(self, node):
        a = self.starts[node.lineno - 1] + node.col_offset
        b = self.starts[node.end_lineno - 1] + node.end_col_offset
        return a, b

    def mk(self, kind, a, b, children=(), fields=None):
        return _TSNode(kind, a, b, self.point(a), self.point(b), children, fields)

    def ident_after(self, a, name, kw):
        i = self.data.find(kw, a) + len(kw)
        i = self.data.find(name.encode(), i)
        return self.mk("identifier", i, i + len(name.encode()))

    def span(self, kind, kids):
        kids = [k for k in kids if k is not None]
        if not kids:
            return None
        return self.mk(kind, min(k.start_byte for k in kids), max(k.end_byte for k in kids), kids)

    def conv(self, n):
        if n is None:
            return None
        if isinstance(n, (_ast.FunctionDef, _ast.AsyncFunctionDef, _ast.ClassDef)):
            a, b = self.pos(n)
            is_cls = isinstance(n, _ast.ClassDef)
            name = self.ident_after(a, n.name, b"class" if is_cls else b"def")
            if is_cls:
                args = self.span("argument_list", [self.conv(x) for x in n.bases + n.keywords])
                kids = [name, args, self.span("block", [self.conv(x) for x in n.body])]
                node = self.mk("class_definition", a, b, [k for k in kids if k is not None])
            else:
                ar = n.args
                params = [self.conv(x) for x in ar.posonlyargs + ar.args + ([ar.vararg] if ar.vararg else [])
                          + ar.kwonlyargs + ([ar.kwarg] if ar.kwarg else [])]
                params += [self.conv(x) for x in ar.defaults + [d for d in ar.kw_defaults if d is not None]]
                kids = [name, self.span("parameters", params), self.conv(n.returns),
                        self.span("block", [self.conv(x) for x in n.body])]
                node = self.mk("function_definition", a, b, [k for k in kids if k is not None])
            if n.decorator_list:
                decs = [self.mk("decorator", *self.pos(d), [self.conv(d)]) for d in n.decorator_list]
                return self.mk("decorated_definition", decs[0].start_byte, b, decs + [node])
            return node
        if isinstance(n, _ast.Import):
            return self.mk("import_statement", *self.pos(n))
        if isinstance(n, _ast.ImportFrom):
            return self.mk("import_from_statement", *self.pos(n))
        if isinstance(n, _ast.Call):
            fn = self.conv(n.func)
            args = self.span("argument_list", [self.conv(x) for x in n.args + n.keywords])
            a, b = self.pos(n)
            return self.mk("call", a, b, [k for k in (fn, args) if k is not None],
                           {"function": fn, "arguments": args})
        if isinstance(n, _ast.Name):
            return self.mk("identifier", *self.pos(n))
        if isinstance(n, _ast.arg):
            a = self.starts[n.lineno - 1] + n.col_offset
            ident = self.mk("identifier", a, a + len(n.arg.encode()))
            ann = self.conv(n.annotation)
            return ident if ann is None else self.span("typed_parameter", [ident, ann])
        if isinstance(n, _ast.Attribute):
            a, b = self.pos(n)
            attr = self.mk("identifier", b - len(n.attr.encode()), b)
            return self.mk("attribute", a, b, [self.conv(n.value), attr])
        if isinstance(n, _ast.keyword):
            val = self.conv(n.value)
            if n.arg is None:
                return self.span("dictionary_splat", [val])
            a = self.starts[n.lineno - 1] + n.col_offset
            return self.span("keyword_argument", [self.mk("identifier", a, a + len(n.arg.encode())), val])
        if isinstance(n, _ast.Lambda):
            a, b = self.pos(n)
            ar = n.args
            params = [self.conv(x) for x in ar.posonlyargs + ar.args + ar.kwonlyargs]
            kids = [self.span("lambda_parameters", params), self.conv(n.body)]
            return self.mk("lambda", a, b, [k for k in kids if k is not None])
        kids = [self.conv(c) for c in _ast.iter_child_nodes(n)]
        kids = [k for k in kids if k is not None]
        if hasattr(n, "lineno") and getattr(n, "end_lineno", None) is not None:
            return self.mk("x_" + type(n).__name__.lower(), *self.pos(n), kids)
        return self.span("x_" + type(n).__name__.lower(), kids)


def structure_python_file(seed, n_units=30):
    """A seeded Python file with the constructs the structure rules care
    about: imports at the top and nested in if/try/classes, decorated and async
    functions, nested classes and functions, methods calling each other,
    attribute / chained / keyword / lambda calls, comments and blank runs."""
    rng = np.random.default_rng(seed)
    names = [f"f{u}" for u in range(n_units)]
    L = ["", "# header comment", "", "import os", "import sys as _sys", "from typing import (", "    List,",
         "    Dict,", ")", "try:", "    import json", "except ImportError:", "    json = None", "",
         "if _sys.version_info >= (3, 8):", "    from functools import cache", "else:",
         "    def cache(f):", "        return f", ""]
    for u in range(n_units):
        r = rng.random()
        callee = names[int(rng.integers(0, n_units))]
        other = names[int(rng.integers(0, n_units))]
        if r < 0.25:
            L += ([f"@cache"] if u % 2 else []) + [f"def {names[u]}(a, b=len('x'), *args, k=None, **kw):",
                                                   f"    \"\"\"Doc {u}.\"\"\"",
                                                   f"    x = {callee}(a, b) + obj.{other}(k=k)",
                                                   f"    return (lambda q: {callee}(q))(x)", ""]
        elif r < 0.45:
            L += [f"class C{u}(Base{u % 3}, metaclass=Meta):", f"    attr = {callee}(1)",
                  "    import re", f"    def {names[u]}(self):", f"        return self.{other}()",
                  "", f"    @property", f"    def p{u}(self):", f"        return {callee}(self)[0]",
                  f"    class Inner{u}:", f"        def {other}(self, x):",
                  f"            return C{u}.{names[u]}(x).{callee}()", ""]
        elif r < 0.6:
            L += [f"async def {names[u]}(x):", f"    await {callee}(x)", f"    def inner_{u}():",
                  f"        return {other}()", f"    return inner_{u}()", ""]
        elif r < 0.8:
            L += [f"RESULT_{u} = {callee}({other}(1), key=lambda v: v)", "", "", f"# comment {u}"]
        else:
            L += [f"for i in range({u}):", f"    {callee}(i)", "", "with open('f') as fh:",
                  f"    def {names[u]}(z):", f"        return {other}(z)", ""]
    L += ["", "if __name__ == '__main__':", f"    {names[0]}(1, 2)", "", ""]
    return "\n".join(L)


def record_structure():
    """TreeSitterSegmenter.segment_code and CrossReferenceAnalyzer.analyze on
    seeded Python files, through the ast-backed stand-in parser."""
    import reference_graph as RG
    import semantic_chunker as SC
    SC.get_parser = lambda lang: _AstAsTreeSitter()
    RG.get_parser = lambda lang: _AstAsTreeSitter()
    out = {}
    files = [("s0", structure_python_file(60)), ("s1", structure_python_file(61, 45)),
             ("s2", synthetic_python_file(62)[0]), ("s3", "\n\n\ndef only():\n    return only()\n\n\n")]
    for name, code in files:
        chunks = SC.TreeSitterSegmenter().segment_code(code, language="python")
        refs = RG.CrossReferenceAnalyzer(chunks, code, language="python").analyze()
        rows = sorted((r.source_chunk_idx, r.target_chunk_idx, r.line_number, r.name) for r in refs)
        out.update({f"{name}_code": np.asarray(code), **{f"{name}_{k}": v for k, v in chunk_arrays(chunks).items()},
                    f"{name}_start": np.asarray([c.start for c in chunks], np.int64),
                    f"{name}_end": np.asarray([c.end for c in chunks], np.int64),
                    f"{name}_parent": np.asarray([c.parent_name or "" for c in chunks]),
                    f"{name}_text": np.asarray([c.text for c in chunks]),
                    f"{name}_ref_src": np.asarray([r[0] for r in rows], np.int32),
                    f"{name}_ref_dst": np.asarray([r[1] for r in rows], np.int32),
                    f"{name}_ref_line": np.asarray([r[2] for r in rows], np.int32),
                    f"{name}_ref_name": np.asarray([r[3] for r in rows])})
        if name in ("s0", "s1"):
            # build_block_indices on the raw source, the structure coming from
            # the segmenter and analyser above (language "python": special
            # lines are on).
            tok = HashTokenizer(vocab=128)
            L = len(tok(code)["input_ids"])
            params = dict(window_size=32, num_prefix_tokens=8, num_suffix_tokens=24, block_size=16,
                          global_last_k_chunks=1, max_chunk_tokens=64)
            R.TreeSitterSegmenter, R.CrossReferenceAnalyzer = SC.TreeSitterSegmenter, RG.CrossReferenceAnalyzer
            R._GLOBAL_CHUNK_CACHE.clear()
            mb = R.StructureAwareMaskBuilder(tok, **params)
            _, bc, bm = mb.build_block_indices(code, L, torch.device("cpu"), language="python")
            out.update({f"{name}_seq_len": np.asarray(L), f"{name}_block_mask": bm.numpy().astype(np.uint8),
                        f"{name}_block_counts": bc.numpy(),
                        **{f"{name}_p_{k}": np.asarray(v) for k, v in params.items()}})
        print(f"structure {name}: lines {code.count(chr(10)) + 1} chunks {len(chunks)} refs {len(rows)}")
    out["files"] = np.asarray([f for f, _ in files])
    np.savez_compressed(os.path.join(HERE, "structure.npz"), **out)


def main():
    base = dict(window_size=192, num_prefix_tokens=64, num_suffix_tokens=128, block_size=64,
                global_last_k_chunks=0, max_chunk_tokens=128)
    cases = [
        # name, L, seed, params-override, tokenizer
        ("c0_4096", 4096, 0, {}, "line"),
        ("c1_12288", 12288, 1, {}, "line"),
        ("c3_16384", 16384, 3, {}, "line"),
        ("ragged_1000", 1000, 5, dict(window_size=64, num_prefix_tokens=4, num_suffix_tokens=300,
                                      global_last_k_chunks=2, max_chunk_tokens=0), "line"),
        ("tiny_40", 40, 6, dict(window_size=0, num_prefix_tokens=0, num_suffix_tokens=0,
                                global_last_k_chunks=1, max_chunk_tokens=0), "line"),
        ("blk128_3000", 3000, 7, dict(block_size=128, window_size=384, max_chunk_tokens=256,
                                      num_suffix_tokens=5000, global_last_k_chunks=3), "line"),
        ("blk128_16384", 16384, 4, dict(block_size=128, window_size=384, num_suffix_tokens=128), "line"),
        ("mct256_2047", 2047, 8, dict(max_chunk_tokens=256, window_size=100, num_prefix_tokens=200), "line"),
        ("words_900", 900, 9, dict(window_size=64, global_last_k_chunks=2), "word"),
    ]
    for name, L, seed, over, tk in cases:
        ss = make_spans(L, seed)
        code = spans_to_code(ss)
        chunks = chunks_from_spanset(ss)
        deps = {int(k): set(int(x) for x in v) for k, v in ss.deps.items()}
        if name == "ragged_1000":
            # out-of-range ids are skipped by the reference (:1530, :1537, :1551)
            deps.setdefault(0, set()).update({len(chunks) + 5, -1})
            deps[len(chunks) + 2] = {0}
            imports = set(ss.import_chunks) | {len(chunks) + 1}
        else:
            imports = set(ss.import_chunks)
        if tk == "word":
            code = "\n".join(" ".join(f"w{j}" for j in range(1 + (i % 3))) for i in range(L))
            L = 900  # tokens (lines have 1-3 words + one special token)
        params = dict(base)
        params.update(over)
        record_mask(name, code=code, seq_len=L, chunks=chunks, deps=deps, imports=imports, language=None,
                    tok=LineTokenizer() if tk == "line" else WordTokenizer(), params=params)
    code, chunks = synthetic_python_file(11)
    params = dict(base)
    params.update(window_size=64, num_prefix_tokens=16, num_suffix_tokens=32, global_last_k_chunks=1)
    L = 700
    imports = {i for i, c in enumerate(chunks) if c.chunk_type == ChunkType.IMPORT}
    record_mask("pyspecial", code=code, seq_len=L, chunks=chunks, deps={}, imports=imports, language="python",
                tok=WordTokenizer(), params=dict(params, block_size=16, max_chunk_tokens=32))
    record_builder_full()
    record_attention("b64", B=2, H=1, L=200, D=128, block=64, seed=21)
    record_attention("b128", B=1, H=1, L=300, D=128, block=128, seed=22)
    record_sparsity_utils()
    record_similarity()
    record_token_level("lines_900", 900, 31, {}, LineTokenizer())
    record_token_level("groups_1000", 1000, 32, dict(max_chunk_tokens=128, window_size=100, global_last_k_chunks=0),
                       LineTokenizer())
    record_token_level("pyspecial_700", 700, 11, dict(num_prefix_tokens=8), WordTokenizer(), language="python")
    record_token_level("attn_256", 256, 33, dict(window_size=16, global_last_k_chunks=0, num_suffix_tokens=8),
                       LineTokenizer(), attn_heads=1)
    record_crossfile()
    record_structure()


if __name__ == "__main__":
    # No recorder named: every fixture. Otherwise the named recorders only, e.g.
    # "python tests/golden/gen_golden.py --reference PATH crossfile".
    _names, _skip = [], False
    for _a in sys.argv[1:]:
        if _skip:
            _skip = False
        elif _a == "--reference":
            _skip = True
        elif not _a.startswith("--reference="):
            _names.append(_a)
    if _names:
        for _n in _names:
            globals()[f"record_{_n}"]()
    else:
        main()
