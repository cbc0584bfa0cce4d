"""Structure-aware block-sparse attention: mask builder and attention module.

Drop-in counterpart of methods/sabrecoder/sabrecoder_attention_triton.py.
Same class and function names, constructor arguments, validation errors and
return types; the arithmetic runs in libsabre_b200.so on the GPU:

* ``StructureAwareMaskBuilder`` (reference :229-1828): text-level work stays
  on the host (tokenizer offsets -> lines -> chunks, signature and special
  lines); the block mask (rules R0-R3, :1455-1604) and the index lists
  (:1837-1859) are built by CUDA kernels.
* ``compute_block_indices_from_mask`` (:1837-1859): CUDA kernel; rows are
  ascending (the reference's unstable argsort leaves them unordered; counts
  and per-row sets are identical).
* ``StructureAwareSparseAttention`` (:1890-2072): same dispatch as the
  reference's ``forward``; the sparse path calls the tcgen05 prefill kernel.
  Optional ``topk_blocks`` adds, per layer and head, the top-k key blocks by
  pooled q.k (no reference counterpart).

Tree-sitter segmentation and the reference graph (semantic_chunker.py,
reference_graph.py) are pluggable: pass ``segmenter_factory`` /
``analyzer_factory`` (same interfaces as the reference classes) or call the
``*_from_chunks`` / ``*_from_spans`` entry points with ready-made structure.
Without them, the reference's tree-sitter modules are used when importable,
else the built-in Python segmenter and analyser of
:mod:`sabrecoder_b200.structure`.
"""

from __future__ import annotations

import math
import re
from collections import OrderedDict
from dataclasses import replace
from typing import Dict, Iterable, List, Optional, Sequence, Set, Tuple

import numpy as np
import torch
import torch.nn as nn

from . import kernels as K
from .chunks import SIGNATURE_TYPES, ChunkType, CodeChunk, type_name

_GLOBAL_CHUNK_CACHE: "OrderedDict" = OrderedDict()
_GLOBAL_LINE_TO_TOKEN_CACHE: "OrderedDict" = OrderedDict()
_GLOBAL_MASK_CACHE: "OrderedDict" = OrderedDict()
_BLOCK_MASK_CACHE: "OrderedDict" = OrderedDict()
_GLOBAL_SIM_VEC_CACHE: "OrderedDict" = OrderedDict()
_GLOBAL_SIM_EDGES_CACHE: "OrderedDict" = OrderedDict()
_GLOBAL_CACHE_MAX_SIZE = 50


def _cache_put(cache: OrderedDict, key, value, cap: int = _GLOBAL_CACHE_MAX_SIZE) -> None:
    if key in cache:
        cache.move_to_end(key)
    cache[key] = value
    while len(cache) > cap:
        cache.popitem(last=False)


def _char_to_line(code: str) -> np.ndarray:
    lens = np.fromiter((len(s) + 1 for s in code.split("\n")), dtype=np.int64)
    return np.repeat(np.arange(1, lens.shape[0] + 1, dtype=np.int64), lens)


def _token_starts(enc, seq_len: int) -> np.ndarray:
    offs = enc.get("offset_mapping")
    ids = enc.get("input_ids")
    if offs is None or ids is None:
        raise RuntimeError("Tokenizer must support return_offsets_mapping and return input_ids for token mapping.")
    n = min(seq_len, len(ids))
    st = np.full(n, -1, dtype=np.int64)
    for t in range(n):
        s = offs[t][0]
        if s is not None and s >= 0:
            st[t] = s
    return st


# A retrieved-segment header of a cross-file prompt: "# <path>: <start> - <end>"
# (Python) or "// <path>: <start> - <end>" (Java), the prompt format the
# reference's evaluator reads (sabrecoder_attention_triton.py:927-935).
_SEGMENT_HEADER = re.compile(r"(#|//)\s+.+:\s*\d+\s*-\s*\d+\s*")


def crossfile_segments(crossfile_code: str) -> List[Tuple[int, int, str]]:
    """``(start_line, end_line, text)`` of each retrieved segment of a
    cross-file context, 1-based inclusive lines (reference :926-985). A
    segment runs from its header line to the line before the next header; a
    span of lines before the first header is a segment of its own. Blank-only
    spans never become segments: they join the segment before them, or the
    first one after them when none precedes."""
    lines = crossfile_code.split("\n")
    heads = [i for i, ln in enumerate(lines, start=1)
             if ln.rstrip().startswith(("# ", "// ")) and _SEGMENT_HEADER.fullmatch(ln.rstrip())]
    if heads:
        spans = ([(1, heads[0] - 1)] if heads[0] > 1 else []) + \
                [(a, b - 1) for a, b in zip(heads, heads[1:] + [len(lines) + 1])]
    else:
        spans = [(1, len(lines))]
    out: List[List[int]] = []
    lead: Optional[int] = None  # first line of blank spans seen before any segment
    for s, e in spans:
        if e < s:
            continue
        if not any(lines[i - 1].strip() for i in range(s, e + 1)):
            if out:
                out[-1][1] = max(out[-1][1], e)
            elif lead is None:
                lead = s
            continue
        if lead is not None:
            s, lead = min(s, lead), None
        out.append([s, e])
    return [(s, e, "\n".join(lines[s - 1 : e])) for s, e in out]


def bits_from_indices(block_indices: torch.Tensor, block_counts: torch.Tensor, ncols: int) -> torch.Tensor:
    """Row bitsets (int32 words, uint32 semantics) from index lists
    ``[..., max]`` + counts ``[...]``: entries below the count in ``[0, ncols)``."""
    idx = block_indices.long()
    ar = torch.arange(idx.shape[-1], device=idx.device)
    ok = (ar < block_counts.long().unsqueeze(-1)) & (idx >= 0) & (idx < ncols)
    nwords = (ncols + 31) // 32
    m = torch.zeros(idx.shape[:-1] + (nwords * 32 + 1,), dtype=torch.bool, device=idx.device)
    m.scatter_(-1, torch.where(ok, idx, torch.full_like(idx, nwords * 32)), True)
    m = m[..., : nwords * 32].reshape(idx.shape[:-1] + (nwords, 32)).to(torch.int64)
    w = (m << torch.arange(32, device=idx.device, dtype=torch.int64)).sum(-1)
    return torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)


class StructureAwareMaskBuilder:
    """Block mask / index-list builder (reference
    sabrecoder_attention_triton.py:229-1828)."""

    def __init__(self, tokenizer, window_size=64, num_prefix_tokens=128, num_suffix_tokens=256,
                 block_size: int = 64, global_last_k_chunks: int = 2, max_chunk_tokens: int = 0,
                 embedding_weight: Optional[torch.Tensor] = None, use_chunk_similarity: bool = False,
                 chunk_similarity_top_percent: float = 0.1, chunk_similarity_max_tokens_per_chunk: int = 256,
                 chunk_similarity_max_neighbors: int = 8, use_crossfile_chunk_similarity: bool = False,
                 crossfile_chunk_similarity_top_percent: Optional[float] = None, *,
                 device: Optional[torch.device] = None, segmenter_factory=None, analyzer_factory=None):
        self.tokenizer = tokenizer
        self.window_size = window_size
        self.num_prefix_tokens = num_prefix_tokens
        self.num_suffix_tokens = num_suffix_tokens
        self.block_size = int(block_size)
        self.global_last_k_chunks = int(global_last_k_chunks)
        self.max_chunk_tokens = int(max_chunk_tokens)
        self.embedding_weight = embedding_weight
        self.use_chunk_similarity = bool(use_chunk_similarity)
        self.chunk_similarity_top_percent = float(chunk_similarity_top_percent)
        self.chunk_similarity_max_tokens_per_chunk = int(chunk_similarity_max_tokens_per_chunk)
        self.chunk_similarity_max_neighbors = int(chunk_similarity_max_neighbors)
        self.use_crossfile_chunk_similarity = bool(use_crossfile_chunk_similarity)
        self.crossfile_chunk_similarity_top_percent = (
            float(crossfile_chunk_similarity_top_percent) if crossfile_chunk_similarity_top_percent is not None
            else float(chunk_similarity_top_percent))
        self.device = device
        self.segmenter_factory = segmenter_factory
        self.analyzer_factory = analyzer_factory
        self.last_block_bits: Optional[torch.Tensor] = None
        # Validation mirrors sabrecoder_attention_triton.py:268-292.
        if self.block_size <= 0:
            raise ValueError("block_size must be > 0.")
        if self.global_last_k_chunks < 0:
            raise ValueError("global_last_k_chunks must be >= 0.")
        if self.max_chunk_tokens < 0:
            raise ValueError("max_chunk_tokens must be >= 0.")
        if self.max_chunk_tokens > 0 and (self.max_chunk_tokens % self.block_size) != 0:
            raise ValueError("max_chunk_tokens must be a multiple of block_size to align with kernel blocks.")
        if self.use_crossfile_chunk_similarity and not self.use_chunk_similarity:
            raise ValueError("use_crossfile_chunk_similarity=True requires use_chunk_similarity=True.")
        if self.use_chunk_similarity:
            if self.embedding_weight is None:
                raise ValueError("use_chunk_similarity=True requires embedding_weight "
                                 "(model.get_input_embeddings().weight).")
            if self.chunk_similarity_top_percent < 0.0:
                raise ValueError("chunk_similarity_top_percent must be >= 0.")
            if self.chunk_similarity_max_tokens_per_chunk <= 0:
                raise ValueError("chunk_similarity_max_tokens_per_chunk must be > 0.")
            if self.chunk_similarity_max_neighbors < 0:
                raise ValueError("chunk_similarity_max_neighbors must be >= 0.")
            if self.use_crossfile_chunk_similarity and self.crossfile_chunk_similarity_top_percent < 0.0:
                raise ValueError("crossfile_chunk_similarity_top_percent must be >= 0.")

    # ------------------------------------------------------------------
    # Host text processing (reference :407-456, :697-858)
    # ------------------------------------------------------------------
    def _encode(self, code: str, seq_len: int):
        return self.tokenizer(code, add_special_tokens=True, truncation=True, max_length=seq_len,
                              return_offsets_mapping=True)

    def _get_token_to_line_mapping(self, code: str, seq_len: int) -> List[int]:
        """Token -> 1-based line, 0 for tokens without an offset (:407-447)."""
        key = (hash(code), seq_len)
        hit = _GLOBAL_LINE_TO_TOKEN_CACHE.get(key)
        if hit is not None:
            return hit
        starts = _token_starts(self._encode(code, seq_len), seq_len)
        c2l = _char_to_line(code)
        out = np.zeros(seq_len, dtype=np.int64)
        ok = starts >= 0
        out[: starts.shape[0]][ok] = c2l[np.minimum(starts[ok], c2l.shape[0] - 1)]
        res = out.tolist()
        _cache_put(_GLOBAL_LINE_TO_TOKEN_CACHE, key, res)
        return res

    def _map_lines_to_tokens(self, code: str, line_numbers: set, seq_len: int) -> torch.Tensor:
        """bool [seq_len]: token lies on one of ``line_numbers`` (:449-456)."""
        if not line_numbers:
            return torch.zeros(seq_len, dtype=torch.bool)
        t2l = np.asarray(self._get_token_to_line_mapping(code, seq_len))
        lines = np.fromiter(line_numbers, dtype=np.int64)
        return torch.from_numpy(np.isin(t2l, lines))

    def _identify_special_lines(self, code: str, chunks, language: Optional[str] = None) -> dict:
        """Python-only globally visible lines (:697-752): module-level
        assignments, type aliases, ``self.x =`` in ``__init__``, returns."""
        empty = {"global_vars": set(), "type_aliases": set(), "class_attrs": set(), "return_stmts": set()}
        if language is None or str(language).lower() not in {"python", "py"}:
            return empty
        fc: Set[int] = set()
        init: Set[int] = set()
        for ch in chunks:
            tn = type_name(ch.chunk_type)
            if tn in SIGNATURE_TYPES:
                fc.update(range(ch.start_line, ch.end_line + 1))
            if tn == "METHOD" and getattr(ch, "name", "") == "__init__":
                init.update(range(ch.start_line, ch.end_line + 1))
        res = {k: set() for k in empty}
        assign = re.compile(r"^[A-Za-z_][A-Za-z0-9_]*\s*[:\[]?\s*=")
        alias = re.compile(r"^[A-Z][A-Za-z0-9_]*\s*=\s*[A-Z][A-Za-z0-9_]*\[")
        attr = re.compile(r"^\s*self\.[A-Za-z_][A-Za-z0-9_]*\s*=")
        ret = re.compile(r"^\s*return\b")
        skip = ("==", "!=", "<=", ">=", "def ", "class ", "import ", "from ")
        for n, line in enumerate(code.split("\n"), start=1):
            s = line.strip()
            if not s or s.startswith("#"):
                continue
            if n not in fc and "=" in s and not any(w in s for w in skip) and assign.match(s):
                res["global_vars"].add(n)
            if "TypeAlias" in s or alias.match(s):
                res["type_aliases"].add(n)
            if n in init and attr.match(line):
                res["class_attrs"].add(n)
            if n in fc and ret.match(s):
                res["return_stmts"].add(n)
        return res

    def _append_uncovered_line_chunks(self, code: str, chunks: List) -> List:
        """Append MODULE_CODE chunks for maximal runs of lines no chunk covers
        (:754-805); existing chunk indices stay stable."""
        if not code:
            return chunks
        lines = code.split("\n")
        n = len(lines)
        if n <= 0:
            return chunks
        covered = np.zeros(n + 1, dtype=bool)
        for ch in chunks or []:
            s = max(1, int(getattr(ch, "start_line", 1) or 1))
            e = min(n, int(getattr(ch, "end_line", 0) or 0))
            if e >= s:
                covered[s : e + 1] = True
        out = list(chunks or [])
        ln = 1
        while ln <= n:
            if covered[ln]:
                ln += 1
                continue
            s = ln
            while ln <= n and not covered[ln]:
                ln += 1
            text = "\n".join(lines[s - 1 : ln - 1])
            out.append(CodeChunk(ChunkType.MODULE_CODE, 0, len(text), text, "", None, s, ln - 1, None, None))
        return out

    def _map_tokens_to_chunks(self, code: str, chunks, seq_len: int) -> List[int]:
        """Token -> chunk through lines; the last chunk in list order wins for a
        line (:807-858)."""
        t2c = np.full(seq_len, -1, dtype=np.int64)
        if not chunks:
            return t2c.tolist()
        nl = len(code.split("\n"))
        l2c = np.full(nl + 1, -1, dtype=np.int64)
        for ci, ch in enumerate(chunks):
            s, e = int(ch.start_line), int(ch.end_line)
            if s >= 0:
                if s <= min(e, nl):
                    l2c[s : min(e, nl) + 1] = ci
            else:  # negative line numbers index from the end, as Python lists do
                for ln in range(s, e + 1):
                    if ln <= nl:
                        l2c[ln] = ci
        enc = self._encode(code, seq_len)
        offs, ids = enc.get("offset_mapping"), enc.get("input_ids")
        if offs is None or ids is None:
            raise RuntimeError("Tokenizer must support return_offsets_mapping and return input_ids for token mapping.")
        if len(offs) < len(ids):
            raise RuntimeError("Tokenizer returned offset_mapping shorter than input_ids; cannot build stable mapping.")
        if not ids:
            return t2c.tolist()
        starts = _token_starts(enc, seq_len)
        c2l = _char_to_line(code)
        ok = starts >= 0
        lines = c2l[np.minimum(starts[ok], c2l.shape[0] - 1)]
        head = t2c[: starts.shape[0]]
        vals = np.where(lines < l2c.shape[0], l2c[np.minimum(lines, l2c.shape[0] - 1)], head[ok])
        head[ok] = vals
        return t2c.tolist()

    # ------------------------------------------------------------------
    # Token-level structure -> GPU
    # ------------------------------------------------------------------
    def structure_to_tokens(self, *, code: str, seq_len: int, chunks: Sequence, chunk_deps: Dict[int, Set[int]],
                            import_chunks: Iterable[int], language: Optional[str]):
        """Host arrays for the mask kernel: token_to_chunk int32[L], global
        token mask uint8[L], chunk flags uint8[nchunks], dependency CSR."""
        t2c = np.asarray(self._map_tokens_to_chunks(code, chunks, seq_len), dtype=np.int32)
        vis: Set[int] = set()
        for ch in chunks:
            if type_name(ch.chunk_type) in SIGNATURE_TYPES:
                s0 = getattr(ch, "signature_start_line", None)
                s1 = getattr(ch, "signature_end_line", None)
                if s0 and s1:
                    vis.update(range(s0, s1 + 1))
        sp = self._identify_special_lines(code, chunks, language=language)
        for key in ("global_vars", "type_aliases", "class_attrs", "return_stmts"):
            vis |= sp[key]
        gtm = self._map_lines_to_tokens(code, vis, seq_len).numpy().astype(np.uint8)
        n = len(chunks)
        flags = np.zeros(n, dtype=np.uint8)
        for c in import_chunks or ():
            c = int(c)
            if 0 <= c < n:
                flags[c] |= 1
        ptr, idx = deps_to_csr(chunk_deps, n)
        return t2c, gtm, flags, ptr, idx

    def build_block_mask_tokens(self, token_to_chunk, chunk_flags, dep_ptr, dep_idx, global_token_mask, seq_len,
                                device=None) -> Tuple[torch.Tensor, torch.Tensor]:
        """GPU block mask from token-level structure: ``(bits, dense)``."""
        dev = torch.device(device if device is not None else (self.device or "cuda"))

        def up(a, dt):
            if isinstance(a, torch.Tensor):
                return a.to(device=dev, dtype=dt, non_blocking=True).contiguous()
            return torch.as_tensor(np.ascontiguousarray(a), dtype=dt).to(dev, non_blocking=True)

        return K.build_block_mask(
            up(token_to_chunk, torch.int32), up(chunk_flags, torch.uint8), up(dep_ptr, torch.int32),
            up(dep_idx, torch.int32), None if global_token_mask is None else up(global_token_mask, torch.uint8),
            seq_len=int(seq_len), block_size=self.block_size, window_size=int(self.window_size),
            num_prefix_tokens=int(self.num_prefix_tokens), num_suffix_tokens=int(self.num_suffix_tokens),
            max_chunk_tokens=self.max_chunk_tokens, global_last_k_chunks=self.global_last_k_chunks)

    def _build_block_mask_from_chunks(self, *, code: str, seq_len: int, chunks: List,
                                      chunk_deps: Dict[int, Set[int]], import_chunks: Set[int],
                                      language: Optional[str], device=None) -> torch.Tensor:
        """int32 ``[nb, nb]`` block mask on the GPU (reference :1455-1604)."""
        t2c, gtm, flags, ptr, idx = self.structure_to_tokens(code=code, seq_len=seq_len, chunks=chunks,
                                                             chunk_deps=chunk_deps, import_chunks=import_chunks,
                                                             language=language)
        bits, dense = self.build_block_mask_tokens(t2c, flags, ptr, idx, gtm, seq_len, device)
        self.last_block_bits = bits
        return dense

    # ------------------------------------------------------------------
    # Index lists
    # ------------------------------------------------------------------
    def _indices_from_bits(self, bits: torch.Tensor, nb: int, batch_size: int):
        idx, cnt, mx = K.indices_from_bits(bits, nb)
        ma = int(mx.item())
        bi = idx[:, :ma].unsqueeze(0).expand(int(batch_size), -1, -1).contiguous()
        bc = cnt.unsqueeze(0).expand(int(batch_size), -1).contiguous()
        return bi, bc

    def build_block_indices_from_chunks(self, code: str, seq_len: int, device, *, chunks: List,
                                        chunk_deps: Dict[int, Set[int]], import_chunks: Set[int],
                                        language: Optional[str] = None, batch_size: int = 1):
        """Index lists for given chunks and dependency edges; with
        ``use_chunk_similarity`` the similarity edges are merged in first
        (without changing the caller's dict), as the reference does (:1798-1805)."""
        if self.use_chunk_similarity:
            sim = self._similarity_edges(chunks, code)
            if sim:
                merged = {k: set(v) for k, v in (chunk_deps or {}).items()}
                for src, tgts in sim.items():
                    merged.setdefault(src, set()).update(tgts)
                chunk_deps = merged
        dense = self._build_block_mask_from_chunks(code=code, seq_len=seq_len, chunks=chunks, chunk_deps=chunk_deps,
                                                   import_chunks=import_chunks, language=language, device=device)
        bi, bc = self._indices_from_bits(self.last_block_bits, dense.shape[0], batch_size)
        return bi, bc, dense

    def build_block_indices_from_spans(self, spanset, device=None, *, batch_size: int = 1):
        """Index lists for seeded synthetic spans (token-level structure, no
        text or tokenizer needed)."""
        ptr, idx = spanset.deps_csr()
        flags = np.asarray([1 if s.tag == "import" else 0 for s in spanset.spans], dtype=np.uint8)
        bits, dense = self.build_block_mask_tokens(spanset.token_to_chunk(), flags, ptr, idx,
                                                   spanset.signature_token_mask(), spanset.seq_len, device)
        self.last_block_bits = bits
        bi, bc = self._indices_from_bits(bits, dense.shape[0], batch_size)
        return bi, bc, dense

    def build_block_indices(self, code: str, seq_len: int, device, *, batch_size: int = 1,
                            crossfile_code: Optional[str] = None, current_code: Optional[str] = None,
                            language: Optional[str] = None, crossfile_full_attention: bool = True):
        """``(block_indices int32 [B, nb, max_active], block_counts int32 [B, nb],
        block_mask_2d int32 [nb, nb])`` on ``device`` (reference :1606-1819)."""
        if crossfile_code is not None and current_code is not None:
            hit = self._crossfile_structure(code, crossfile_code, current_code, language, crossfile_full_attention)
            dense = self._build_block_mask_from_chunks(code=code, seq_len=seq_len, chunks=hit["chunks"],
                                                       chunk_deps=hit["chunk_deps"],
                                                       import_chunks=hit["import_chunks"], language=language,
                                                       device=device)
            bi, bc = self._indices_from_bits(self.last_block_bits, dense.shape[0], batch_size)
            return bi, bc, dense
        hit = self._structure_for_code(code, language)
        return self.build_block_indices_from_chunks(code, seq_len, device, chunks=hit["chunks"],
                                                    chunk_deps=hit["chunk_deps"], import_chunks=hit["import_chunks"],
                                                    language=language, batch_size=batch_size)

    def _structure_for_code(self, code: str, language: Optional[str]) -> Dict:
        """Chunks, dependency edges and import chunks of a prompt from the
        segmenter and reference analyser (cached per prompt), the gaps filled
        with line chunks (reference :1774-1797)."""
        key = (hash(code), str(language).lower() if language else None)
        hit = _GLOBAL_CHUNK_CACHE.get(key)
        if hit is None:
            seg, ana = self._structure_backends()
            chunks = seg(tokenizer=self.tokenizer).segment_code(code, language=language)
            imports = {i for i, c in enumerate(chunks) if type_name(c.chunk_type) == "IMPORT"}
            deps: Dict[int, Set[int]] = {}
            for ref in ana(chunks, code, language=language).analyze():
                s_, t_ = ref.source_chunk_idx, ref.target_chunk_idx
                deps.setdefault(s_, set()).add(t_)
                deps.setdefault(t_, set()).add(s_)
            chunks = self._append_uncovered_line_chunks(code, chunks)
            hit = {"chunks": chunks, "chunk_deps": deps, "import_chunks": imports}
            _cache_put(_GLOBAL_CHUNK_CACHE, key, hit)
        return hit

    def _crossfile_structure(self, code: str, crossfile_code: str, current_code: str, language: Optional[str],
                             full_attention: bool) -> Dict:
        """Chunks of a cross-file prompt ``code = crossfile_code + current
        file`` (reference :1622-1772 and :872-1040), similarity edges included:

        * the retrieved context becomes one globally visible chunk
          (``full_attention``) or one chunk per retrieved segment
          (:func:`crossfile_segments`);
        * the current file is segmented and analysed on its own, its gaps
          filled with line chunks, its lines shifted by the context's line count
          and its chunk ids by the context's chunk count;
        * with ``use_chunk_similarity``, current-file chunks link to their most
          similar context chunks, and with ``use_crossfile_chunk_similarity``
          context chunks link among themselves at
          ``crossfile_chunk_similarity_top_percent``."""
        if not code.startswith(crossfile_code):
            raise ValueError("full_code does not start with crossfile_code; dataset fields are inconsistent.")
        shift = len(crossfile_code.split("\n")) if crossfile_code else 0
        chunks: List = []
        global_chunks: Set[int] = set()
        if crossfile_code and crossfile_code.strip():
            if full_attention:
                chunks.append(CodeChunk(ChunkType.MODULE_CODE, 0, len(crossfile_code), crossfile_code, "", None,
                                        1, shift, None, None))
                global_chunks.add(0)
            else:
                for s, e, text in crossfile_segments(crossfile_code):
                    chunks.append(CodeChunk(ChunkType.MODULE_CODE, 0, len(text), text, "", None, s, e, None, None))
        ncf = len(chunks)
        deps: Dict[int, Set[int]] = {}
        imports: Set[int] = set()
        if current_code and current_code.strip():
            seg, ana = self._structure_backends()
            cur = seg(tokenizer=self.tokenizer).segment_code(current_code, language=language)
            for c in self._append_uncovered_line_chunks(current_code, cur):
                chunks.append(replace(
                    c, start_line=c.start_line + shift, end_line=c.end_line + shift,
                    signature_start_line=(c.signature_start_line + shift) if c.signature_start_line else None,
                    signature_end_line=(c.signature_end_line + shift) if c.signature_end_line else None))
            # Analyser ids index the segmenter's own list, which the gap
            # chunks extend at the end, so shifting by ncf keeps them valid.
            for ref in ana(cur, current_code, language=language).analyze():
                s_, t_ = ref.source_chunk_idx + ncf, ref.target_chunk_idx + ncf
                deps.setdefault(s_, set()).add(t_)
                deps.setdefault(t_, set()).add(s_)
            imports = {i + ncf for i, c in enumerate(cur) if type_name(c.chunk_type) == "IMPORT"}
        if self.use_chunk_similarity:
            sim = self._similarity_edges(chunks, code, src_indices=list(range(ncf, len(chunks))),
                                         tgt_indices=list(range(ncf)))
            for s_, tg in sim.items():
                deps.setdefault(s_, set()).update(tg)
            if self.use_crossfile_chunk_similarity and ncf > 1:
                cf = list(range(ncf))
                sim = self._similarity_edges(chunks, code, src_indices=cf, tgt_indices=cf,
                                             top_percent=self.crossfile_chunk_similarity_top_percent)
                for s_, tg in sim.items():
                    deps.setdefault(s_, set()).update(tg)
        return {"chunks": chunks, "chunk_deps": deps, "import_chunks": imports | global_chunks}

    # ------------------------------------------------------------------
    # Token-level variant (reference :1171-1454, :1862-1885)
    # ------------------------------------------------------------------
    def token_rule_arrays(self, *, code: str, seq_len: int, chunks: Sequence, chunk_deps: Dict[int, Set[int]],
                          import_chunks: Iterable[int], language: Optional[str]):
        """Host arrays of the token-level rule: ``(chunk int32[L], group
        int32[L], global uint8[L], dependency bits uint32[nchunks, words],
        nchunks)``. Raises like the reference when fewer than 10 % of the
        tokens map to a chunk (:1256-1264)."""
        t2c, gtm, flags, ptr, idx = self.structure_to_tokens(code=code, seq_len=seq_len, chunks=chunks,
                                                             chunk_deps=chunk_deps, import_chunks=import_chunks,
                                                             language=language)
        L, n = int(seq_len), len(chunks)
        valid = t2c >= 0
        nvalid = int(valid.sum())
        ratio = nvalid / L if L > 0 else 0.0
        if ratio < 0.1:
            raise RuntimeError(f"Token-to-chunk mapping ratio too low ({ratio:.3f}). seq_len={L}, "
                               f"valid_mappings={nvalid}, num_chunks={n}")
        glob = gtm.astype(bool)
        if n > 0:
            glob |= valid & (flags[np.clip(t2c, 0, n - 1)] & 1).astype(bool)
            k = int(self.global_last_k_chunks)
            if k > 0:
                glob |= valid & (t2c >= max(0, n - k))
        npre = min(int(self.num_prefix_tokens), L)
        if npre > 0:
            glob[:npre] = True
        nsuf = min(int(self.num_suffix_tokens), L)
        if nsuf > 0:
            glob[max(0, L - nsuf):] = True
        if self.max_chunk_tokens > 0:
            bpg = max(1, self.max_chunk_tokens // self.block_size)
            gidx = (np.arange(L) // self.block_size) // bpg
            ng = int(gidx.max()) + 2 if L > 0 else 2
            grp = t2c.astype(np.int64) * ng + gidx
            if n * ng >= 2 ** 31:
                raise ValueError("too many chunk groups for 32-bit group ids")
        else:
            grp = t2c
        words = max((n + 31) // 32, 1)
        dep = np.zeros((max(n, 1), words), dtype=np.uint32)
        for s_ in range(n):
            for t_ in idx[ptr[s_]:ptr[s_ + 1]]:
                dep[s_, int(t_) >> 5] |= np.uint32(1 << (int(t_) & 31))
        return t2c, grp.astype(np.int32), glob.astype(np.uint8), dep, n

    def build_token_level_blocks(self, code: str, seq_len: int, device, *, chunks: Sequence,
                                 chunk_deps: Dict[int, Set[int]], import_chunks: Iterable[int],
                                 language: Optional[str] = None, batch_size: int = 1,
                                 merge_similarity: bool = True):
        """Token-level variant without an L x L mask: ``(block_indices [B, nb,
        max_active], block_counts [B, nb], block_mask_2d [nb, nb], (tile_masks
        int64 [n_listed, 64], row_ptr int32 [nb]))`` on ``device``. The lists
        are the blocks holding any visible pair (the reference's block mask of
        the token mask), ascending; the tile masks hold each listed block's
        64 query rows' key bits, in list order. Block size 64.
        ``merge_similarity=False`` takes ``chunk_deps`` as final (the
        cross-file path has merged its own similarity edges)."""
        if self.block_size != 64:
            raise ValueError("the token-level variant uses block_size 64")
        if self.use_chunk_similarity and merge_similarity:
            sim = self._similarity_edges(chunks, code)
            if sim:
                merged = {k: set(v) for k, v in (chunk_deps or {}).items()}
                for src, tgts in sim.items():
                    merged.setdefault(src, set()).update(tgts)
                chunk_deps = merged
        t2c, grp, glob, dep, n = self.token_rule_arrays(code=code, seq_len=seq_len, chunks=chunks,
                                                        chunk_deps=chunk_deps, import_chunks=import_chunks,
                                                        language=language)
        dev = torch.device(device if device is not None else (self.device or "cuda"))

        def up(a, dt):
            return torch.as_tensor(np.ascontiguousarray(a), dtype=dt).to(dev)

        tc, tg, tgl = up(t2c, torch.int32), up(grp, torch.int32), up(glob, torch.uint8)
        db = up(dep.view(np.int32), torch.int32)
        w = int(self.window_size)
        bits = K.token_block_mask(tc, tg, tgl, db, n, w)
        nb = bits.shape[0]
        idx, cnt, mx = K.indices_from_bits(bits, nb)
        ma = max(int(mx.item()), 1)
        lists = idx[:, :ma].contiguous()
        masks, row_ptr = K.token_tile_masks(tc, tg, tgl, db, n, w, lists, cnt)
        shifts = torch.arange(32, device=dev, dtype=torch.int32)
        dense = ((bits.unsqueeze(-1) >> shifts) & 1).reshape(nb, -1)[:, :nb].to(torch.int32).contiguous()
        self.last_block_bits = bits
        bi = lists.unsqueeze(0).expand(int(batch_size), -1, -1).contiguous()
        bc = cnt.unsqueeze(0).expand(int(batch_size), -1).contiguous()
        return bi, bc, dense, (masks, row_ptr)

    def build_token_level_mask(self, code: str, seq_len: int, device, dtype, crossfile_code: Optional[str] = None,
                               current_code: Optional[str] = None, language: Optional[str] = None,
                               crossfile_full_attention: bool = True) -> torch.Tensor:
        """The reference's dense ``(L, L)`` mask, 0 where visible and -inf
        elsewhere (:1269-1454), expanded from the per-block tile masks. O(L^2)
        memory: a debugging and compatibility helper; the attention path keeps
        only the listed blocks' masks."""
        if crossfile_code is not None and current_code is not None:
            hit = self._crossfile_structure(code, crossfile_code, current_code, language, crossfile_full_attention)
        else:
            hit = self._structure_for_code(code, language)
        bi, bc, _, (masks, row_ptr) = self.build_token_level_blocks(
            code, seq_len, device, chunks=hit["chunks"], chunk_deps=hit["chunk_deps"],
            import_chunks=hit["import_chunks"], language=language,
            merge_similarity=crossfile_code is None or current_code is None)
        return expand_token_masks(bi[0], bc[0], masks, int(seq_len), dtype)

    # ------------------------------------------------------------------
    # Chunk-similarity edges (reference :458-682)
    # ------------------------------------------------------------------
    @staticmethod
    def _clean_for_similarity(text: str) -> str:
        """Drop a leading "# " or "// " from every line: cross-file context is
        stored as commented code and the comment marks should not dominate
        the embedding (reference :458-472)."""
        out = []
        for ln in text.split("\n"):
            if ln.startswith("# "):
                out.append(ln[2:])
            elif ln.startswith("// "):
                out.append(ln[3:])
            else:
                out.append(ln)
        return "\n".join(out)

    def _similarity_token_lists(self, texts: List[str]) -> List[List[int]]:
        """One batched tokenizer call with truncation and padding (ids where the
        attention mask is set); a tokenizer without that interface is called
        per text through ``encode`` (reference :526-554)."""
        cap = int(self.chunk_similarity_max_tokens_per_chunk)
        try:
            enc = self.tokenizer(texts, add_special_tokens=False, truncation=True, max_length=cap, padding=True,
                                 return_tensors="pt")
            ids, am = enc.get("input_ids", None), enc.get("attention_mask", None)
            if ids is None or am is None:
                raise RuntimeError("tokenizer returned no input_ids/attention_mask")
            ids = torch.as_tensor(ids).cpu().numpy()
            am = torch.as_tensor(am).cpu().numpy().astype(bool)
            return [ids[r][am[r]].tolist() for r in range(ids.shape[0])]
        except Exception:  # noqa: BLE001 -- same fallback as the reference
            return [list(self.tokenizer.encode(t, add_special_tokens=False))[:cap] if t and t.strip() else []
                    for t in texts]

    def _device_embedding(self) -> torch.Tensor:
        emb = self.embedding_weight
        if emb is None:
            raise RuntimeError("embedding_weight is required for chunk similarity but is None.")
        if emb.is_cuda:
            return emb.detach()
        dev = self.device if self.device is not None and torch.device(self.device).type == "cuda" else "cuda"
        key = ("emb", emb.data_ptr(), tuple(emb.shape), str(emb.dtype), str(dev))
        hit = _GLOBAL_SIM_VEC_CACHE.get(key)
        if hit is None:
            hit = emb.detach().to(dev)
            _cache_put(_GLOBAL_SIM_VEC_CACHE, key, hit)
        return hit

    def _get_or_build_similarity_vectors(self, chunks: List, code: str) -> Tuple[torch.Tensor, List[int]]:
        """``(vectors fp16 [M, D] on the GPU, idx_map)``: one unit vector per
        chunk whose cleaned text is not blank, ``idx_map[row]`` its chunk index
        (reference :490-579). Vectors come from sabre_chunk_vectors."""
        emb = self._device_embedding()
        tok_key = getattr(self.tokenizer, "name_or_path", None) or type(self.tokenizer).__name__
        key = (hash(code), tok_key, int(self.chunk_similarity_max_tokens_per_chunk), str(emb.device),
               str(emb.dtype), int(emb.data_ptr()))
        hit = _GLOBAL_SIM_VEC_CACHE.get(key)
        if hit is not None:
            return hit[0], list(hit[1])
        texts, idx_map = [], []
        for i, c in enumerate(chunks):
            cleaned = self._clean_for_similarity(getattr(c, "text", "") or "")
            if cleaned and cleaned.strip():
                texts.append(cleaned)
                idx_map.append(i)
        if not texts:
            mat = torch.empty(0, emb.shape[1], dtype=torch.float16, device=emb.device)
        else:
            lists = self._similarity_token_lists(texts)
            vocab = emb.shape[0]
            for ids in lists:
                if any(t < 0 or t >= vocab for t in ids):
                    raise IndexError(f"token id outside the embedding table of {vocab} rows")
            ptr = np.zeros(len(lists) + 1, dtype=np.int32)
            ptr[1:] = np.cumsum([len(x) for x in lists])
            flat = np.asarray([t for x in lists for t in x], dtype=np.int32)
            mat = K.chunk_vectors(emb, torch.from_numpy(ptr).to(emb.device),
                                  torch.from_numpy(flat).to(emb.device))
        _cache_put(_GLOBAL_SIM_VEC_CACHE, key, (mat, list(idx_map)))
        return mat, list(idx_map)

    def _similarity_edges(self, chunks: List, code: str, *, src_indices: Optional[List[int]] = None,
                          tgt_indices: Optional[List[int]] = None,
                          top_percent: Optional[float] = None) -> Dict[int, Set[int]]:
        """Directed edges {source chunk: {target chunks}}: each source's
        ``k = min(max_neighbors, floor(top_frac * num_targets))`` most similar
        targets, itself excluded (reference :581-682). Exact score ties go to
        the lower target position."""
        if not self.use_chunk_similarity:
            return {}
        frac = float(self.chunk_similarity_top_percent) if top_percent is None else float(top_percent)
        if frac > 1.0:  # a percentage
            frac /= 100.0
        frac = max(0.0, min(1.0, frac))
        if self.chunk_similarity_max_neighbors <= 0 or frac <= 0.0:
            return {}
        src = list(range(len(chunks))) if src_indices is None else list(src_indices)
        tgt = list(range(len(chunks))) if tgt_indices is None else list(tgt_indices)
        key = (hash(code), frac, self.chunk_similarity_max_tokens_per_chunk, self.chunk_similarity_max_neighbors,
               hash(tuple(src)), hash(tuple(tgt)))
        hit = _GLOBAL_SIM_EDGES_CACHE.get(key)
        if hit is not None:
            return {k: set(v) for k, v in hit.items()}
        mat, idx_map = self._get_or_build_similarity_vectors(chunks, code)
        edges: Dict[int, Set[int]] = {}
        row_of = {c: r for r, c in enumerate(idx_map)}
        sr = [(c, row_of[c]) for c in src if c in row_of]
        tg = [(c, row_of[c]) for c in tgt if c in row_of]
        k = min(int(self.chunk_similarity_max_neighbors), int(math.floor(len(tg) * frac))) if tg else 0
        if sr and tg and k > 0:
            dev = mat.device

            def i32(xs):
                return torch.tensor(xs, dtype=torch.int32, device=dev)

            picks = K.similarity_topk(mat, i32([r for _, r in sr]), i32([c for c, _ in sr]),
                                      i32([r for _, r in tg]), i32([c for c, _ in tg]), k).cpu().numpy()
            for (c, _), row in zip(sr, picks):
                for t in row:
                    if t >= 0:
                        edges.setdefault(int(c), set()).add(int(t))
        _cache_put(_GLOBAL_SIM_EDGES_CACHE, key, {k_: set(v) for k_, v in edges.items()})
        return edges

    def _structure_backends(self):
        """Segmenter and analyser classes: the ones passed to the constructor,
        else the reference's tree-sitter modules when importable, else the
        built-in ones: Python on the ``ast`` tree (:mod:`sabrecoder_b200.structure`),
        Java and C# on a token stream (:mod:`sabrecoder_b200.structure_braces`)."""
        seg, ana = self.segmenter_factory, self.analyzer_factory
        if seg is None or ana is None:
            try:
                from semantic_chunker import TreeSitterSegmenter  # the reference's segmenter, if importable
                from reference_graph import CrossReferenceAnalyzer
            except Exception:  # noqa: BLE001  (tree-sitter not installed)
                from .structure_braces import StructureAnalyzer as CrossReferenceAnalyzer
                from .structure_braces import StructureSegmenter as TreeSitterSegmenter
            seg = seg or TreeSitterSegmenter
            ana = ana or CrossReferenceAnalyzer
        return seg, ana

    def clear_cache(self):
        clear_all_caches()


def expand_token_masks(indices: torch.Tensor, counts: torch.Tensor, tile_masks: torch.Tensor, seq_len: int,
                       dtype=torch.float32) -> torch.Tensor:
    """Dense ``(L, L)`` 0/-inf mask from listed blocks' 64-bit row masks."""
    dev = indices.device
    nb = indices.shape[0]
    Lp = nb * 64
    out = torch.full((nb, 64, nb, 64), float("-inf"), dtype=dtype, device=dev)
    cnt = counts.long()
    rows = torch.repeat_interleave(torch.arange(nb, device=dev), cnt)
    pos = torch.arange(int(cnt.sum().item()), device=dev) - torch.repeat_interleave(torch.cumsum(cnt, 0) - cnt, cnt)
    cols = indices.long()[rows, pos]
    shifts = torch.arange(64, device=dev, dtype=torch.int64)
    bits = ((tile_masks[: rows.numel()].unsqueeze(-1) >> shifts) & 1).bool()  # [n, 64 rows, 64 keys]
    blk = out[rows, :, cols, :]
    blk[bits] = 0
    out[rows, :, cols, :] = blk
    return out.reshape(Lp, Lp)[:seq_len, :seq_len].contiguous()


def deps_to_csr(chunk_deps: Optional[Dict[int, Iterable[int]]], nchunks: int):
    """Dependency dict -> CSR (dep_ptr int32[nchunks+1], dep_idx int32[]),
    dropping out-of-range sources and targets (the reference skips them,
    :1530 and :1537)."""
    ptr = np.zeros(nchunks + 1, dtype=np.int32)
    flat: List[int] = []
    deps = chunk_deps or {}
    for c in range(nchunks):
        tg = deps.get(c)
        if tg:
            flat.extend(sorted(int(t) for t in tg if 0 <= int(t) < nchunks))
        ptr[c + 1] = len(flat)
    return ptr, np.asarray(flat, dtype=np.int32)


def compute_block_indices_from_mask(block_mask: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """``(block_indices int32 [B, nb, max_active], block_counts int32 [B, nb])``
    from a ``[B, nb_m, nb_n]`` mask (reference :1837-1859). Runs on the GPU;
    CPU inputs are moved there and the results moved back."""
    dev = block_mask.device
    m = block_mask if block_mask.is_cuda else block_mask.to("cuda")
    idx, cnt, mx = K.indices_from_dense(m)
    ma = int(mx.item())
    bi = idx[..., :ma].contiguous()
    return bi.to(dev), cnt.to(dev)


def compute_block_mask_from_token_mask(token_mask: torch.Tensor, block_size_m: int, block_size_n: int) -> torch.Tensor:
    """Block (i, j) is active iff any token pair in it is not -inf
    (reference :1862-1885). O(L^2) debugging helper; plain torch ops."""
    L = token_mask.shape[0]
    nbm = (L + block_size_m - 1) // block_size_m
    nbn = (L + block_size_n - 1) // block_size_n
    pm, pn = nbm * block_size_m - L, nbn * block_size_n - L
    if pm or pn:
        token_mask = torch.nn.functional.pad(token_mask, (0, pn, 0, pm), value=float("-inf"))
    t = token_mask.view(nbm, block_size_m, nbn, block_size_n)
    return (~torch.isinf(t)).any(dim=(1, 3)).to(torch.int32)


class StructureAwareSparseAttention(nn.Module):
    """Attention module (reference StructureAwareSparseAttentionTriton,
    :1890-2072). ``forward(q, k, v, code=...)`` takes ``[B, H, L, D]`` tensors
    (any strides with unit head-dim stride; K/V may have fewer heads)."""

    def __init__(self, tokenizer, block_size=64, window_size=64, num_prefix_tokens=128, num_suffix_tokens=256,
                 use_token_level_sparsity=False, embedding_weight: Optional[torch.Tensor] = None,
                 global_last_k_chunks: int = 2, max_chunk_tokens: int = 0, use_chunk_similarity: bool = False,
                 chunk_similarity_top_percent: float = 0.1, chunk_similarity_max_tokens_per_chunk: int = 256,
                 chunk_similarity_max_neighbors: int = 8, use_crossfile_chunk_similarity: bool = False,
                 crossfile_chunk_similarity_top_percent: Optional[float] = None, topk_blocks: int = 0,
                 segmenter_factory=None, analyzer_factory=None):
        super().__init__()
        if use_token_level_sparsity and int(block_size) != 64:
            raise ValueError("use_token_level_sparsity=True needs block_size=64")
        if use_token_level_sparsity and int(topk_blocks) > 0:
            raise ValueError("the pooled top-k extension is not combined with token-level sparsity")
        self.tokenizer = tokenizer
        self.block_size = int(block_size)
        self.window_size = window_size
        self.num_prefix_tokens = num_prefix_tokens
        self.num_suffix_tokens = num_suffix_tokens
        self.use_token_level_sparsity = bool(use_token_level_sparsity)
        self.topk_blocks = int(topk_blocks)
        self._bits_cache = None
        self.mask_builder = StructureAwareMaskBuilder(
            tokenizer=tokenizer, block_size=self.block_size, window_size=window_size,
            num_prefix_tokens=num_prefix_tokens, num_suffix_tokens=num_suffix_tokens,
            global_last_k_chunks=global_last_k_chunks, max_chunk_tokens=max_chunk_tokens,
            embedding_weight=embedding_weight, use_chunk_similarity=use_chunk_similarity,
            chunk_similarity_top_percent=chunk_similarity_top_percent,
            chunk_similarity_max_tokens_per_chunk=chunk_similarity_max_tokens_per_chunk,
            chunk_similarity_max_neighbors=chunk_similarity_max_neighbors,
            use_crossfile_chunk_similarity=use_crossfile_chunk_similarity,
            crossfile_chunk_similarity_top_percent=crossfile_chunk_similarity_top_percent,
            segmenter_factory=segmenter_factory, analyzer_factory=analyzer_factory)

    def _lookup_blocks(self, query, code, batch_size):
        from .sabrecoder_llama import get_precomputed_blocks
        gi, gc = get_precomputed_blocks()
        if gi is not None and gc is not None:
            return gi, gc
        mb = self.mask_builder
        key = (hash(code), query.shape[2], self.block_size, query.device, batch_size, mb.window_size,
               mb.num_prefix_tokens, mb.num_suffix_tokens, mb.block_size, mb.global_last_k_chunks,
               mb.max_chunk_tokens, mb.use_chunk_similarity)
        hit = _BLOCK_MASK_CACHE.get(key)
        if hit is None:
            bi, bc, _ = mb.build_block_indices(code, query.shape[2], query.device, batch_size=batch_size)
            hit = (bi, bc)
            _cache_put(_BLOCK_MASK_CACHE, key, hit)
        return hit

    def _lookup_token_blocks(self, query, code, batch_size):
        """Token-level lists and tile masks of a prompt (cached). Precomputed
        block-level lists are not needed here: every visible token pair lies in
        a block the token rule lists."""
        mb = self.mask_builder
        key = ("token", hash(code), query.shape[2], query.device, batch_size, mb.window_size, mb.num_prefix_tokens,
               mb.num_suffix_tokens, mb.global_last_k_chunks, mb.max_chunk_tokens, mb.use_chunk_similarity)
        hit = _BLOCK_MASK_CACHE.get(key)
        if hit is None:
            st = mb._structure_for_code(code, None)
            bi, bc, _, tm = mb.build_token_level_blocks(code, query.shape[2], query.device, chunks=st["chunks"],
                                                        chunk_deps=st["chunk_deps"],
                                                        import_chunks=st["import_chunks"], batch_size=batch_size)
            hit = (bi, bc, tm)
            _cache_put(_BLOCK_MASK_CACHE, key, hit)
        return hit

    def forward(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, code: str = None,
                attention_mask: Optional[torch.Tensor] = None,
                precomputed_block_indices: Optional[torch.Tensor] = None,
                precomputed_block_counts: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                pooled: Optional[Tuple[torch.Tensor, torch.Tensor]] = None) -> torch.Tensor:
        B, H, Lq, D = query.shape
        Lk = key.shape[2]
        if code is not None and Lq == Lk and Lq > 1 and self.use_token_level_sparsity:
            bi, bc, tm = self._lookup_token_blocks(query, code, B)
            return K.prefill_bsa(query, key, value, bi, bc, self.block_size, out=out, token_masks=tm)
        if code is not None and Lq == Lk and Lq > 1:
            if precomputed_block_indices is not None and precomputed_block_counts is not None:
                bi, bc = precomputed_block_indices, precomputed_block_counts
            else:
                bi, bc = self._lookup_blocks(query, code, B)
            if self.topk_blocks > 0:
                bi, bc = self.extend_topk(query, key, bi, bc, pooled=pooled)
            return K.prefill_bsa(query, key, value, bi, bc, self.block_size, out=out)
        # Dense path for everything else, as the reference does (:2056-2066).
        if attention_mask is not None and attention_mask.shape[-2:] != (Lq, Lk):
            attention_mask = None
        if key.shape[1] != H:
            g = H // key.shape[1]
            key = key.repeat_interleave(g, dim=1)
            value = value.repeat_interleave(g, dim=1)
        return torch.nn.functional.scaled_dot_product_attention(
            query, key, value, attn_mask=attention_mask, dropout_p=0.0, is_causal=attention_mask is None)

    def extend_topk(self, query, key, block_indices, block_counts, pooled=None):
        """Per-head lists: structure rows plus the top-k blocks by pooled q.k.
        ``pooled`` may carry the per-block means already computed (by the fused
        RoPE kernel); otherwise they are computed here."""
        L = query.shape[2]
        nb = (L + self.block_size - 1) // self.block_size
        base = block_indices[0] if block_indices.dim() == 3 else block_indices[0, 0]
        cnt = block_counts[0] if block_counts.dim() == 2 else block_counts[0, 0]
        # Every layer of a forward sees the same list tensors; their bitset is
        # built once (the cache holds the tensors, so identity stays valid).
        c = self._bits_cache
        if c is None or c[0] is not block_indices or c[1] is not block_counts or c[2] != nb:
            c = (block_indices, block_counts, nb, bits_from_indices(base, cnt, nb))
            self._bits_cache = c
        bits = c[3]
        if pooled is not None:
            qm, km = pooled
        else:
            qm = K.pool_blocks(query, self.block_size)
            km = K.pool_blocks(key, self.block_size)
        idx, c, mx, _ = K.topk_extend(qm, km, bits, self.topk_blocks,
                                      cap=min(nb, block_indices.shape[-1] + self.topk_blocks))
        return idx, c

    def clear_cache(self):
        self.mask_builder.clear_cache()


def get_cache_stats() -> Dict[str, int]:
    stats = {
        "chunk_cache_size": len(_GLOBAL_CHUNK_CACHE),
        "line_to_token_cache_size": len(_GLOBAL_LINE_TO_TOKEN_CACHE),
        "mask_cache_size": len(_GLOBAL_MASK_CACHE),
        "block_mask_cache_size": len(_BLOCK_MASK_CACHE),
        "sim_edges_cache_size": 0,
        "sim_vec_cache_size": 0,
    }
    stats["total_cached_items"] = sum(stats.values())
    return stats


def print_cache_stats() -> None:
    s = get_cache_stats()
    print("\n" + "=" * 60 + "\nCACHE STATISTICS\n" + "=" * 60)
    for k, v in s.items():
        print(f"  {k:32s} {v:3d}")
    print("=" * 60 + "\n")


def clear_all_caches() -> None:
    for c in (_GLOBAL_CHUNK_CACHE, _GLOBAL_LINE_TO_TOKEN_CACHE, _GLOBAL_MASK_CACHE, _BLOCK_MASK_CACHE,
              _GLOBAL_SIM_VEC_CACHE, _GLOBAL_SIM_EDGES_CACHE):
        c.clear()


# Names the reference uses for the same objects.
StructureAwareSparseAttentionTriton = StructureAwareSparseAttention
