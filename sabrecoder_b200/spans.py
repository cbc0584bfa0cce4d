"""Seeded synthetic code-structure spans.

The reference derives chunks from tree-sitter segmentation of real source files
(methods/sabrecoder/semantic_chunker.py:125-170) and call/inherit edges from a
name-based reference graph (methods/sabrecoder/reference_graph.py:196-266).
Neither tree-sitter nor the evaluation datasets exist on the machines this
library is built and measured on, so prompts are stood in for by seeded spans
with the shapes those components produce:

* spans cover the prompt contiguously; lengths are uniform in [min_len, max_len]
  tokens;
* each span is tagged ``import`` / ``class`` / ``function`` / ``statement``
  (``statement`` maps to ``MODULE_CODE``); imports only occur in a header
  region at the start of the prompt, as they do in real files;
* class and function spans carry a one-line signature on their first line;
* call edges join function spans to earlier function/class spans, and are
  symmetrised exactly as the reference's callers do
  (methods/sabrecoder/sabrecoder_attention_triton.py:1786-1789).

One token maps to one line (token ``t`` is line ``t + 1``), so a span given in
tokens is also a span in lines.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Set

import numpy as np

# Chunk type codes shared with the C-ABI (include/sabre_b200.h).
CHUNK_IMPORT = 0
CHUNK_FUNCTION = 1
CHUNK_CLASS = 2
CHUNK_METHOD = 3
CHUNK_MODULE_CODE = 4

TAG_TO_TYPE = {
    "import": CHUNK_IMPORT,
    "function": CHUNK_FUNCTION,
    "class": CHUNK_CLASS,
    "statement": CHUNK_MODULE_CODE,
}


@dataclass
class Span:
    tag: str
    start: int  # first token (inclusive)
    end: int    # last token (inclusive)

    @property
    def chunk_type(self) -> int:
        return TAG_TO_TYPE[self.tag]

    @property
    def has_signature(self) -> bool:
        return self.tag in ("class", "function")


@dataclass
class SpanSet:
    seq_len: int
    spans: List[Span]
    deps: Dict[int, Set[int]] = field(default_factory=dict)

    @property
    def import_chunks(self) -> Set[int]:
        return {i for i, s in enumerate(self.spans) if s.tag == "import"}

    def token_to_chunk(self) -> np.ndarray:
        t2c = np.full(self.seq_len, -1, dtype=np.int32)
        for i, s in enumerate(self.spans):
            t2c[s.start : s.end + 1] = i
        return t2c

    def signature_token_mask(self) -> np.ndarray:
        """Tokens on signature lines (first line of every class/function span)."""
        m = np.zeros(self.seq_len, dtype=np.uint8)
        for s in self.spans:
            if s.has_signature:
                m[s.start] = 1
        return m

    def chunk_types(self) -> np.ndarray:
        return np.array([s.chunk_type for s in self.spans], dtype=np.int32)

    def deps_csr(self):
        """Dependency lists as CSR (dep_ptr[nchunks+1], dep_idx[ndeps])."""
        n = len(self.spans)
        ptr = np.zeros(n + 1, dtype=np.int32)
        idx: List[int] = []
        for c in range(n):
            tg = sorted(self.deps.get(c, ()))
            idx.extend(tg)
            ptr[c + 1] = len(idx)
        return ptr, np.asarray(idx, dtype=np.int32)


def make_spans(
    seq_len: int,
    seed: int,
    *,
    min_len: int = 20,
    max_len: int = 400,
    header_frac: float = 0.03,
    p_class: float = 0.06,
    p_function: float = 0.18,
    call_prob: float = 0.5,
    max_calls: int = 2,
) -> SpanSet:
    """Seeded spans covering ``[0, seq_len)``.

    Imports fill the header region (the first ``header_frac`` of the prompt);
    after it each span is a class with probability ``p_class``, a function with
    probability ``p_function``, else a statement span.
    """
    rng = np.random.default_rng(seed)
    spans: List[Span] = []
    header_end = int(seq_len * header_frac)
    pos = 0
    while pos < seq_len:
        n = int(rng.integers(min_len, max_len + 1))
        end = min(seq_len - 1, pos + n - 1)
        if pos < header_end:
            tag = "import"
        else:
            u = rng.random()
            tag = "class" if u < p_class else ("function" if u < p_class + p_function else "statement")
        spans.append(Span(tag, pos, end))
        pos = end + 1
    deps: Dict[int, Set[int]] = {}
    defs = [i for i, s in enumerate(spans) if s.tag in ("class", "function")]
    for j, i in enumerate(defs):
        if spans[i].tag != "function" or j == 0:
            continue
        if rng.random() >= call_prob:
            continue
        for _ in range(int(rng.integers(1, max_calls + 1))):
            tgt = defs[int(rng.integers(0, j))]
            deps.setdefault(i, set()).add(tgt)
            deps.setdefault(tgt, set()).add(i)
    return SpanSet(seq_len, spans, deps)


def spans_to_code(spanset: SpanSet) -> str:
    """One text line per token (the line's content is irrelevant to the mask
    when no language is given; see sabrecoder_attention_triton.py:701-703)."""
    return "\n".join("x" for _ in range(spanset.seq_len))


class LineTokenizer:
    """Tokenizer stand-in: one token per line, with character offsets.

    Provides the interface the reference's token mapping needs
    (``input_ids`` + ``offset_mapping``, sabrecoder_attention_triton.py:824-836).
    """

    name_or_path = "line-tokenizer"

    def __call__(self, code, add_special_tokens=True, truncation=True, max_length=None,
                 return_offsets_mapping=False, **kw):
        offs = []
        pos = 0
        for ln in code.split("\n"):
            offs.append((pos, pos + len(ln)))
            pos += len(ln) + 1
        if max_length is not None:
            offs = offs[:max_length]
        out = {"input_ids": list(range(len(offs)))}
        if return_offsets_mapping:
            out["offset_mapping"] = offs
        return out


class WordTokenizer:
    """Tokenizer stand-in with several tokens per line: splits on spaces and
    newlines, and prepends one special token with offset (0, 0) when
    ``add_special_tokens`` is set (as HF fast tokenizers do for BOS)."""

    name_or_path = "word-tokenizer"

    def __call__(self, code, add_special_tokens=True, truncation=True, max_length=None,
                 return_offsets_mapping=False, **kw):
        offs = [(0, 0)] if add_special_tokens else []
        i = 0
        n = len(code)
        while i < n:
            if code[i] in " \n":
                i += 1
                continue
            j = i
            while j < n and code[j] not in " \n":
                j += 1
            offs.append((i, j))
            i = j
        if truncation and max_length is not None:
            offs = offs[:max_length]
        out = {"input_ids": list(range(len(offs)))}
        if return_offsets_mapping:
            out["offset_mapping"] = offs
        return out


class HashTokenizer:
    """Tokenizer stand-in whose ids depend on the text: words (split on spaces
    and newlines) map to a stable hash modulo ``vocab``. Offers the batched
    call (padding, ``return_tensors="pt"``, attention mask) and ``encode``
    that the chunk-similarity text side uses, plus offsets like
    :class:`WordTokenizer` for the token-to-line mapping."""

    name_or_path = "hash-tokenizer"

    def __init__(self, vocab: int = 512):
        self.vocab = int(vocab)

    def _words(self, text):
        spans = []
        i, n = 0, len(text)
        while i < n:
            if text[i] in " \n":
                i += 1
                continue
            j = i
            while j < n and text[j] not in " \n":
                j += 1
            spans.append((i, j))
            i = j
        return spans

    def _id(self, word: str) -> int:
        h = 2166136261
        for ch in word.encode("utf-8"):
            h = ((h ^ ch) * 16777619) & 0xFFFFFFFF
        return h % self.vocab

    def encode(self, text, add_special_tokens=False, **kw):
        return [self._id(text[a:b]) for a, b in self._words(text)]

    def __call__(self, text, add_special_tokens=True, truncation=True, max_length=None, padding=False,
                 return_tensors=None, return_offsets_mapping=False, **kw):
        def one(t):
            offs = self._words(t)
            ids = [self._id(t[a:b]) for a, b in offs]
            if truncation and max_length is not None:
                ids, offs = ids[:max_length], offs[:max_length]
            return ids, offs

        if isinstance(text, (list, tuple)):
            rows = [one(t)[0] for t in text]
            width = max((len(r) for r in rows), default=0)
            ids = [r + [0] * (width - len(r)) for r in rows]
            mask = [[1] * len(r) + [0] * (width - len(r)) for r in rows]
            if return_tensors == "pt":
                import torch
                return {"input_ids": torch.tensor(ids, dtype=torch.long).reshape(len(rows), width),
                        "attention_mask": torch.tensor(mask, dtype=torch.long).reshape(len(rows), width)}
            return {"input_ids": ids, "attention_mask": mask}
        ids, offs = one(text)
        out = {"input_ids": ids}
        if return_offsets_mapping:
            out["offset_mapping"] = offs
        return out


# Span mix used for the benchmark workloads: structure alone gives about 10-13%
# causal block density at 12K-16K tokens (block 64, 4-block window, sink block,
# 128-token groups), about 15-21% with the pooled top-8 blocks added.
BENCH_SPAN_MIX = dict(p_class=0.03, p_function=0.10, header_frac=0.01)
