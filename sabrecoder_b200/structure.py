"""Code structure for Python prompts without tree-sitter.

The reference segments a prompt with tree-sitter and links chunks by name
(``TreeSitterSegmenter``, methods/sabrecoder/semantic_chunker.py:48-460, and
``CrossReferenceAnalyzer``, methods/sabrecoder/reference_graph.py:160-270).
tree-sitter is an optional native dependency; for Python source the same
rules can be applied to the syntax tree of the standard ``ast`` module, which
is what this module does:

* chunks (semantic_chunker.py:125-267): a pre-order walk that does not enter
  function bodies; every ``import`` / ``from ... import`` statement is an
  IMPORT chunk, a class a CLASS chunk (its body is walked with the class as
  parent), a function a FUNCTION chunk, or a METHOD chunk of the nearest
  enclosing class. A chunk spans its node (``def`` / ``class`` / ``import``
  keyword to the end of its last token; decorators are not part of it), and
  its signature is its first line.
* gaps (semantic_chunker.py:323-453): maximal runs of lines no chunk covers
  become MODULE_CODE chunks; an all-blank run is instead joined to the
  MODULE_CODE chunk that ends right before it, else to the first chunk that
  ends right before it, else to the first chunk that starts right after it
  (such a chunk is rebuilt from whole lines), else it becomes a MODULE_CODE
  chunk too. MODULE_CODE chunks come first in the result.
* references (reference_graph.py:191-250): for every call, the callee name
  is the identifier that ends last inside the called expression (``f`` in
  ``f(x)``, ``m`` in ``a.b(c).m()``); the call's line belongs to the last
  chunk covering it; a reference goes to every other chunk of that name.
  Python classes contribute no inheritance references in the reference.

Source that does not parse as a whole is repaired locally, as tree-sitter
recovers around an error: the line a syntax error is reported on is replaced
by ``pass`` at its indentation and the parse retried (up to ``max_fixes``
times; a Python 2 ``print x`` in the middle of a file then costs that line
only). If that does not converge (a prompt cut in the middle of a
statement), the last lines are dropped one at a time (up to
``max_trim_lines``) and become MODULE_CODE through the gap rule. Chunks next
to a syntax error may differ from tree-sitter's.
"""

from __future__ import annotations

import ast
import threading
from collections import deque
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

from .chunks import ChunkType, CodeChunk

# Language markers, checked in this order (semantic_chunker.py:51-56, :104-123).
_MARKERS = (("c_sharp", ("using System", "namespace ", "public class", "private class")),
            ("java", ("package ", "import java.", "public class", "private class", "public static void")),
            ("python", ("def ", "class ", "import ", "from ")))


def detect_language(code: str) -> str:
    for lang, marks in _MARKERS:
        if any(m in code for m in marks):
            return lang
    return "python"


def _norm_language(language: Optional[str], code: str) -> str:
    if not language:
        return detect_language(code)
    low = language.lower()
    return {"csharp": "c_sharp", "c#": "c_sharp"}.get(low, low)


class _Source:
    """UTF-8 byte offsets of a source string's lines (ast columns are bytes)."""

    def __init__(self, code: str):
        self.code = code
        self.data = code.encode("utf-8", errors="replace")
        self.line_start = [0]
        pos = self.data.find(b"\n")
        while pos >= 0:
            self.line_start.append(pos + 1)
            pos = self.data.find(b"\n", pos + 1)

    def byte(self, lineno: int, col: int) -> int:
        return self.line_start[lineno - 1] + col

    def text(self, a: int, b: int) -> str:
        return self.data[a:b].decode("utf-8", errors="replace")

    def line_span(self, first: int, last: int) -> Tuple[int, int]:
        """Bytes of whole lines first..last (1-based, inclusive, the last
        line's newline included)."""
        n = len(self.line_start)
        first = max(first, 1)
        last = max(last, first)
        a = self.line_start[min(first - 1, n - 1)]
        b = len(self.data) if last >= n else self.line_start[last]
        return a, b


def _neutralised(lines: List[str], max_fixes: int) -> Optional[ast.Module]:
    """Parse, replacing each line a syntax error points at by ``pass``."""
    lines = list(lines)
    for _ in range(max_fixes + 1):
        try:
            return ast.parse("\n".join(lines))
        except SyntaxError as e:
            ln = min(max(int(e.lineno or len(lines)), 1), len(lines))
            body = lines[ln - 1]
            fix = body[: len(body) - len(body.lstrip())] + "pass"
            if body == fix:  # already neutral: the error is not local to this line
                return None
            lines[ln - 1] = fix
        except ValueError:
            return None
    return None


# The segmenter and the analyser parse the same prompt one after the other,
# so each thread keeps its last parse (one entry per thread: a worker thread
# never sees another thread's tree, and at most one prompt's text and tree per
# thread stay alive after the call). Trees returned by _parse are shared by
# both callers and must be treated as read-only.
_PARSE_LOCAL = threading.local()


def clear_parse_cache() -> None:
    """Drop the calling thread's cached parse."""
    _PARSE_LOCAL.entry = None


def _parse(code: str, max_trim_lines: int, max_fixes: int = 64) -> Tuple[Optional[ast.Module], int]:
    """(module, number of trailing lines dropped to make it parse). The
    module is cached for the calling thread and must not be modified."""
    key = (code, max_trim_lines, max_fixes)
    hit = getattr(_PARSE_LOCAL, "entry", None)
    if hit is not None and hit[0] == key:
        return hit[1]
    result: Tuple[Optional[ast.Module], int] = (None, 0)
    lines = code.split("\n")
    for drop in range(0, min(max_trim_lines, len(lines) - 1) + 1):
        tree = _neutralised(lines[: len(lines) - drop], max_fixes if drop == 0 else 0)
        if tree is not None:
            result = (tree, drop)
            break
    _PARSE_LOCAL.entry = (key, result)
    return result


def _calls(tree: ast.AST) -> List[ast.Call]:
    """The Call nodes of a tree in ``ast.walk`` order (breadth first, fields
    in declaration order), without its per-node generators."""
    AST, Call = ast.AST, ast.Call
    out: List[ast.Call] = []
    todo = deque([tree])
    pop, push, extend = todo.popleft, todo.append, todo.extend
    while todo:
        node = pop()
        if node.__class__ is Call:
            out.append(node)
        for name in node._fields:
            v = getattr(node, name, None)
            if v.__class__ is list:
                extend([x for x in v if isinstance(x, AST)])
            elif isinstance(v, AST):
                push(v)
    return out


class PythonSegmenter:
    """Drop-in for ``TreeSitterSegmenter(tokenizer).segment_code(code,
    language)`` on Python source (see the module docstring)."""

    def __init__(self, tokenizer=None, max_trim_lines: int = 64):
        self.tokenizer = tokenizer
        self.max_trim_lines = int(max_trim_lines)

    def segment_code(self, code: str, language: Optional[str] = None) -> List[CodeChunk]:
        if not code or not code.strip():
            return []
        lang = _norm_language(language, code)
        if lang != "python":
            raise ValueError(f"the built-in segmenter handles Python only (got {lang}); install tree-sitter "
                             "or pass segmenter_factory/analyzer_factory")
        src = _Source(code)
        tree, _ = _parse(code, self.max_trim_lines)
        chunks: List[CodeChunk] = []
        if tree is not None:
            self._walk(tree.body, src, None, chunks)
        return self._fill_gaps(src, chunks)

    def _chunk(self, node, src: _Source, kind: ChunkType, name: str, parent: Optional[str]) -> CodeChunk:
        a = src.byte(node.lineno, node.col_offset)
        b = src.byte(node.end_lineno, node.end_col_offset)
        sig = node.lineno if kind in (ChunkType.CLASS, ChunkType.FUNCTION, ChunkType.METHOD) else None
        return CodeChunk(kind, a, b, src.text(a, b), name, parent, node.lineno, node.end_lineno, sig, sig)

    def _walk(self, nodes: Sequence[ast.AST], src: _Source, parent: Optional[str], out: List[CodeChunk]) -> None:
        for node in nodes:
            if isinstance(node, (ast.Import, ast.ImportFrom)):
                out.append(self._chunk(node, src, ChunkType.IMPORT, "import", None))
            elif isinstance(node, ast.ClassDef):
                out.append(self._chunk(node, src, ChunkType.CLASS, node.name, None))
                self._walk(node.body, src, node.name, out)
            elif isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef)):
                kind = ChunkType.METHOD if parent else ChunkType.FUNCTION
                out.append(self._chunk(node, src, kind, node.name, parent))
            elif isinstance(node, ast.stmt):
                # Compound statements (if / for / while / try / with / match):
                # definitions and imports nested in them count too.
                self._walk(_nested_statements(node), src, parent, out)

    @staticmethod
    def _fill_gaps(src: _Source, sem: List[CodeChunk]) -> List[CodeChunk]:
        lines = src.code.split("\n")
        n = len(lines)
        covered = [False] * (n + 2)
        for c in sem:
            for ln in range(max(1, c.start_line or 1), min(n, c.end_line or n) + 1):
                covered[ln] = True

        def whole_lines(c: CodeChunk, first: int, last: int) -> CodeChunk:
            a, b = src.line_span(first, last)
            return CodeChunk(c.chunk_type, a, b, src.text(a, b), c.name or "", c.parent_name, first, last,
                             c.signature_start_line, c.signature_end_line)

        def module(first: int, last: int) -> CodeChunk:
            a, b = src.line_span(first, last)
            return CodeChunk(ChunkType.MODULE_CODE, a, b, src.text(a, b), "", None, first, last, None, None)

        mods: List[CodeChunk] = []
        ln = 1
        while ln <= n:
            if covered[ln]:
                ln += 1
                continue
            first = ln
            while ln <= n and not covered[ln]:
                ln += 1
            last = ln - 1
            if any(lines[k - 1].strip() for k in range(first, last + 1)):
                mods.append(module(first, last))
                continue
            if mods and mods[-1].end_line == first - 1:
                mods[-1] = whole_lines(mods[-1], mods[-1].start_line, last)
                continue
            before = next((i for i, c in enumerate(sem) if c.end_line == first - 1), None)
            if before is not None:
                sem[before] = whole_lines(sem[before], sem[before].start_line, last)
                continue
            after = next((i for i, c in enumerate(sem) if c.start_line == last + 1), None)
            if after is not None:
                sem[after] = whole_lines(sem[after], first, sem[after].end_line)
                continue
            mods.append(module(first, last))
        return mods + sem


def _nested_statements(node: ast.stmt) -> List[ast.stmt]:
    out: List[ast.stmt] = []
    for field in ("body", "orelse", "finalbody"):
        out.extend(getattr(node, field, None) or [])
    for h in getattr(node, "handlers", None) or []:
        out.extend(h.body)
    for case in getattr(node, "cases", None) or []:
        out.extend(case.body)
    # Source order: a try's handlers come before its else and finally.
    out.sort(key=lambda s: (s.lineno, s.col_offset))
    return out


@dataclass
class Reference:
    """Same fields as the reference's ``CrossReference`` (reference_graph.py:23-36)."""

    source_chunk_idx: int
    target_chunk_idx: int
    ref_type: str
    name: str
    line_number: int
    confidence: float = 1.0


def _identifiers(node: ast.AST, src: _Source):
    """(end byte, name) of every identifier token inside an expression."""
    for sub in ast.walk(node):
        if isinstance(sub, ast.Name):
            yield src.byte(sub.end_lineno, sub.end_col_offset), sub.id
        elif isinstance(sub, ast.Attribute):
            yield src.byte(sub.end_lineno, sub.end_col_offset), sub.attr
        elif isinstance(sub, ast.keyword) and sub.arg is not None and hasattr(sub, "lineno"):
            yield src.byte(sub.lineno, sub.col_offset) + len(sub.arg.encode()), sub.arg
        elif isinstance(sub, ast.arg):
            yield src.byte(sub.lineno, sub.col_offset) + len(sub.arg.encode()), sub.arg


class PythonReferenceAnalyzer:
    """Drop-in for ``CrossReferenceAnalyzer(chunks, code, language).analyze()``
    on Python source: call references between chunks by callee name."""

    def __init__(self, chunks, code: str, language: Optional[str] = None, max_trim_lines: int = 64):
        self.chunks = chunks
        self.code = code
        self.language = _norm_language(language, code)
        self.max_trim_lines = int(max_trim_lines)
        self.chunk_by_name: Dict[str, List[int]] = {}
        self.chunk_by_line: Dict[int, int] = {}
        for i, c in enumerate(chunks):
            name = getattr(c, "name", "") or ""
            if name:
                self.chunk_by_name.setdefault(name, []).append(i)
            for ln in range(int(getattr(c, "start_line", 0) or 0), int(getattr(c, "end_line", 0) or 0) + 1):
                self.chunk_by_line[ln] = i
        self.references: List[Reference] = []

    def analyze(self) -> List[Reference]:
        if self.language != "python":
            raise ValueError(f"the built-in analyser handles Python only (got {self.language})")
        src = _Source(self.code)
        tree, _ = _parse(self.code, self.max_trim_lines)
        self.references = []
        if tree is None:
            return self.references
        for node in _calls(tree):
            line = node.lineno
            source = self.chunk_by_line.get(line)
            if source is None:
                continue
            ids = list(_identifiers(node.func, src))
            if not ids:
                continue
            name = max(ids, key=lambda t: t[0])[1]
            for target in self.chunk_by_name.get(name, ()):
                if target != source:
                    self.references.append(Reference(source, target, "call", name, line))
        return self.references
