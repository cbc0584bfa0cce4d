"""Code structure for Java and C# prompts without tree-sitter.

The reference segments Java and C# with tree-sitter grammars
(``TreeSitterSegmenter``, methods/sabrecoder/semantic_chunker.py:48-460, node
types :59-74) and links chunks by name (``CrossReferenceAnalyzer``,
methods/sabrecoder/reference_graph.py:160-270, call node types :198-208,
callee names :87-114, base types :117-157). tree-sitter is not installed
here; this module applies the same rules to a token stream (one regular
expression per language finds comments, strings, text blocks and character
literals, so brackets inside them do not count), with a declaration scanner
that matches brackets:

* chunks -- Java: ``package`` / ``import`` declarations are IMPORT chunks;
  ``class`` / ``interface`` / ``enum`` declarations CLASS chunks whose bodies
  are walked with the class as parent; methods and constructors FUNCTION or
  METHOD chunks (bodies are not walked). ``record`` and ``@interface``
  declarations are no chunks, but their bodies are walked with the outer
  parent. C#: ``using`` directives are IMPORT chunks; ``class`` /
  ``interface`` / ``struct`` CLASS chunks; methods and constructors as in
  Java; namespaces, records and enums are walked without being chunks.
  Methods of anonymous classes created in field initializers are METHOD
  chunks of the enclosing class (the reference walks into field
  declarations). A declaration spans its first modifier, annotation or
  attribute to its closing brace or semicolon; comments before it are not
  part of it. Its signature is its first line.
* names -- the first identifier child of the declaration node, as the
  reference takes it: the declared name, except for a C# method whose return
  type is a plain identifier (``Task Run()`` is named ``Task``, as
  tree-sitter-c-sharp parses that type as an identifier node).
* gaps -- the same rule as the Python segmenter (MODULE_CODE chunks first).
* references -- Java: every method invocation (callee = its name), object
  creation (the last identifier of the whole ``new ...`` expression) and
  ``this(...)`` / ``super(...)`` call (the last identifier in it); C#: every
  invocation (the last identifier of the called expression, generic
  arguments included) and object creation (as in Java). A reference goes
  from the chunk owning the line where the expression starts (the last chunk
  covering it) to every other chunk of that name. Inheritance: a Java class's
  ``extends`` type (its last identifier) and every type identifier of its
  ``implements`` list (Java interfaces give none: their ``extends`` clause is
  not the field the reference reads); every identifier of a C# class /
  interface / struct base list.

Parity is unpinned: tree-sitter's parse (its error recovery in particular)
cannot be run here, so these rules are restated from the reference's code
and the grammars' documented node shapes.
"""

from __future__ import annotations

import bisect
import re
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from .chunks import ChunkType, CodeChunk
from .structure import PythonSegmenter, Reference, _norm_language, _Source

_JAVA_KW = frozenset("""abstract assert boolean break byte case catch char class const continue default do double
else enum extends final finally float for goto if implements import instanceof int interface long native new
package private protected public return short static strictfp super switch synchronized this throw throws
transient try void volatile while true false null var sealed permits yield""".split())
_JAVA_MODS = frozenset("""public protected private static final abstract synchronized native transient volatile
strictfp default sealed non-sealed""".split())
_CS_KW = frozenset("""abstract as base bool break byte case catch char checked class const continue decimal default
delegate do double else enum event explicit extern false finally fixed float for foreach goto if implicit in int
interface internal is lock long namespace new null object operator out override params private protected public
readonly ref return sbyte sealed short sizeof stackalloc static string struct switch this throw true try typeof
uint ulong unchecked unsafe ushort using virtual void volatile while""".split())
_CS_MODS = frozenset("""public private protected internal static readonly sealed override virtual abstract extern
unsafe new async partial const volatile ref required file""".split())
# Names that open a statement or an expression with parentheses, never a call.
_JAVA_NOT_CALLS = frozenset("if for while switch catch synchronized return throw try assert do else case".split())
_CS_NOT_CALLS = frozenset("""if for foreach while switch catch lock using return throw try do else case fixed typeof
sizeof default checked unchecked when""".split())

# One token per match; whitespace, comments and (C#) preprocessor lines are
# matched and dropped. Literals follow the languages' lexical grammars
# (JLS 3.10.5-3.10.6 strings, text blocks and characters; C# regular,
# verbatim, interpolated and raw strings): a literal that is not closed runs
# to the end of its line (the end of the file for text blocks, verbatim and raw
# strings). An interpolated C# string ends at its first unescaped quote, so a
# quote inside one of its {holes} ends it early.
_OPS = r"->|=>|::|\?\?|\?\.|&&|\|\||[<>!=]=|<<|\+\+|--|\S"
_JAVA_LEX = re.compile(
    r'(?P<skip>\s+|//[^\n]*|/\*.*?(?:\*/|\Z))'
    r'|(?P<lit>"""(?:[^"\\]|\\.|"(?!""))*(?:"""|\Z)|"(?:[^"\\\n]|\\.)*"?|\'(?:[^\'\\\n]|\\.)*\'?)'
    r'|(?P<id>@?[^\W\d][\w$]*|\$[\w$]*)'
    r'|(?P<num>\d[\w.]*)'
    r'|(?P<p>' + _OPS + r')', re.S)
_CS_LEX = re.compile(
    r'(?P<skip>\s+|//[^\n]*|/\*.*?(?:\*/|\Z)|\#[^\n]*)'
    r'|(?P<lit>\$*(?P<rq>"{3,}).*?(?:(?P=rq)|\Z)'
    r'|(?:@\$?|\$@)"(?:[^"]|"")*"?'
    r'|\$?"(?:[^"\\\n]|\\.)*"?'
    r"|'(?:[^'\\\n]|\\.)*'?)"
    r'|(?P<id>@?[^\W\d]\w*)'
    r'|(?P<num>\d[\w.]*)'
    r'|(?P<p>' + _OPS + r')', re.S)


@dataclass
class _Tok:
    kind: str  # "id", "kw", "lit", "p" (punctuation / operator)
    text: str
    b0: int    # first byte
    b1: int    # byte after the last
    line: int  # 1-based line of the first byte
    eline: int  # line of the last byte


def _byte_offsets(code: str):
    """Character index -> UTF-8 byte offset (a lone surrogate counts as the
    one byte its replacement character takes); None for ASCII text."""
    if code.isascii():
        return None
    cp = np.frombuffer(code.encode("utf-32-le", errors="surrogatepass"), dtype=np.uint32)
    n = np.where(cp < 0x80, 1, np.where(cp < 0x800, 2, np.where(cp < 0x10000, 3, 4)))
    n[(cp >= 0xD800) & (cp < 0xE000)] = 1
    out = np.zeros(len(code) + 1, dtype=np.int64)
    np.cumsum(n, out=out[1:])
    return out.tolist()


def _tokens(code: str, lang: str) -> List[_Tok]:
    lex = _JAVA_LEX if lang == "java" else _CS_LEX
    kws = _JAVA_KW if lang == "java" else _CS_KW
    boff = _byte_offsets(code)
    nl = [m.start() for m in re.finditer("\n", code)]
    out: List[_Tok] = []
    append = out.append
    bis = bisect.bisect_right
    for m in lex.finditer(code):
        kind = m.lastgroup
        if kind == "skip":
            continue
        s, e = m.span()
        text = m.group()
        if kind == "rq":
            kind = "lit"
        elif kind == "id":
            if text in kws:
                kind = "kw"
        elif kind == "num":
            kind = "lit"
        line = bis(nl, s - 1) + 1
        eline = line if kind != "lit" else bis(nl, e - 2) + 1
        if boff is None:
            append(_Tok(kind, text, s, e, line, eline))
        else:
            append(_Tok(kind, text, boff[s], boff[e], line, eline))
    return out


_OPEN = {"(": ")", "[": "]", "{": "}"}
_CLOSE = {")": "(", "]": "[", "}": "{"}


def _match(toks: Sequence[_Tok], i: int) -> int:
    """Index of the bracket closing toks[i] (or the last token)."""
    depth = 0
    for j in range(i, len(toks)):
        t = toks[j].text
        if t in _OPEN:
            depth += 1
        elif t in _CLOSE:
            depth -= 1
            if depth == 0:
                return j
    return len(toks) - 1


def _match_back(toks: Sequence[_Tok], j: int) -> int:
    """Index of the bracket opening toks[j]."""
    depth = 0
    for i in range(j, -1, -1):
        t = toks[i].text
        if t in _CLOSE:
            depth += 1
        elif t in _OPEN:
            depth -= 1
            if depth == 0:
                return i
    return 0


def _until(toks: Sequence[_Tok], i: int, end: int, stops: Tuple[str, ...]) -> int:
    """First index >= i of a token in ``stops`` outside any bracket (or end)."""
    j = i
    while j < end:
        t = toks[j].text
        if t in stops:
            return j
        if t in _OPEN:
            j = _match(toks, j) + 1
            continue
        j += 1
    return end


class _Scanner:
    """Declarations of a Java or C# token stream (see the module docstring)."""

    def __init__(self, toks: List[_Tok], lang: str):
        self.t = toks
        self.lang = lang
        self.java = lang == "java"
        self.mods = _JAVA_MODS if self.java else _CS_MODS
        self.decl_names: set = set()   # name tokens of methods/constructors/types
        self.classes: List[Tuple[int, int, int]] = []  # (first token, header end, kind: 0 java class, 1 other)
        self.chunks: List[Tuple[ChunkType, int, int, str, Optional[str]]] = []
        self._in_type = False

    # -- helpers -----------------------------------------------------------
    def _skip_prefix(self, i: int, end: int) -> int:
        """Past annotations / attributes / modifiers starting at i."""
        t = self.t
        while i < end:
            x = t[i].text
            if self.java and x.startswith("@") and x != "@" and i + 1 <= end:
                if x == "@interface" or (x == "@" and i + 1 < end and t[i + 1].text == "interface"):
                    return i
                i += 1
                if i < end and t[i].text == "(":
                    i = _match(t, i) + 1
                continue
            if self.java and x == "@" and i + 1 < end and t[i + 1].text != "interface":
                i += 2  # "@ Name" split by the lexer
                while i + 1 < end and t[i].text == "." and t[i + 1].kind == "id":
                    i += 2
                if i < end and t[i].text == "(":
                    i = _match(t, i) + 1
                continue
            if not self.java and x == "[":
                i = _match(t, i) + 1
                continue
            if x in self.mods:
                i += 1
                continue
            return i
        return i

    def _type_kw(self, i: int, h: int) -> int:
        """Index of the type keyword of a declaration header [i, h), or -1."""
        kws = ("class", "interface", "enum", "record") if self.java else (
            "class", "interface", "struct", "record", "enum", "delegate")
        depth = 0
        for j in range(i, h):
            x = self.t[j].text
            if x in _OPEN:
                depth += 1
            elif x in _CLOSE:
                depth -= 1
            elif depth == 0 and (x in kws or (self.java and x == "@interface")):
                if x == "record" and (j + 1 >= h or self.t[j + 1].kind != "id"):
                    continue
                return j
        return -1

    # -- scopes ------------------------------------------------------------
    def scan(self) -> None:
        self._scope(0, len(self.t), None, unit=True)

    def _scope(self, i: int, end: int, parent: Optional[str], unit: bool = False, enum_body: bool = False) -> None:
        t = self.t
        self._in_type = not unit
        if enum_body:
            i = self._enum_constants(i, end, parent)
        while i < end:
            x = t[i].text
            if x == ";":
                i += 1
                continue
            if x == "{":  # initializer block
                i = _match(t, i) + 1
                continue
            if unit and self.java and x in ("package", "import"):
                j = _until(t, i, end, (";",))
                self.chunks.append((ChunkType.IMPORT, i, min(j, end - 1), "import", None))
                i = j + 1
                continue
            if not self.java and (x == "using" or (x == "global" and i + 1 < end and t[i + 1].text == "using")) \
                    and self._using_directive(i, end):
                j = _until(t, i, end, (";",))
                self.chunks.append((ChunkType.IMPORT, i, min(j, end - 1), "import", None))
                i = j + 1
                continue
            if not self.java and x == "namespace":
                j = _until(t, i, end, ("{", ";"))
                if j < end and t[j].text == "{":
                    k = _match(t, j)
                    self._scope(j + 1, k, parent, unit=True)
                    i = k + 1
                else:
                    i = j + 1  # file-scoped: the rest of the file follows at this level
                continue
            i = self._member(i, end, parent)

    def _using_directive(self, i: int, end: int) -> bool:
        j = i + 1 if self.t[i].text == "using" else i + 2
        # "using (" / "using var" are statements (only inside bodies, which are not walked)
        return j < end and self.t[j].text not in ("(",) and not (self.t[j].text == "var")

    def _enum_constants(self, i: int, end: int, parent: Optional[str]) -> int:
        """Java enum body: constants (some with class bodies) up to ';'."""
        t = self.t
        while i < end:
            x = t[i].text
            if x == ";":
                return i + 1
            if x == "(":
                i = _match(t, i) + 1
                continue
            if x == "{":
                k = _match(t, i)
                if self.java:
                    self._scope(i + 1, k, parent)
                    self._in_type = True
                i = k + 1
                continue
            i += 1
        return i

    def _member(self, i: int, end: int, parent: Optional[str]) -> int:
        t = self.t
        p = self._skip_prefix(i, end)
        if p >= end:
            return end
        h = _until(t, p, end, ("{", ";", "=", "=>"))
        tk = self._type_kw(p, h if h < end else end)
        if tk >= 0:
            return self._type_decl(i, tk, end, parent)
        paren = _until(t, p, h, ("(",))
        if paren < h and t[paren].text == "(":
            return self._method(i, p, paren, end, parent)
        return self._field(i, p, end, parent)

    def _type_decl(self, i: int, tk: int, end: int, parent: Optional[str]) -> int:
        t = self.t
        kw = t[tk].text
        name_tok = tk + 1
        while name_tok < end and t[name_tok].kind != "id":
            name_tok += 1
        name = t[name_tok].text if name_tok < end else "unknown"
        j = min(name_tok + 1, end)
        while j < end and t[j].text not in ("{", ";"):
            j = _match(t, j) + 1 if t[j].text in ("(", "[") else j + 1
        if self.java:
            chunk = kw in ("class", "interface", "enum")
        else:
            chunk = kw in ("class", "interface", "struct")
        self.decl_names.add(name_tok)
        if kw in ("class", "interface") or (not self.java and kw == "struct"):
            self.classes.append((i, j, 0 if (self.java and kw == "class") else (2 if self.java else 1)))
        if j < end and t[j].text == "{":
            k = _match(t, j)
            if chunk:
                self.chunks.append((ChunkType.CLASS, i, k, name, None))
            walk_parent = name if chunk else parent
            if kw == "delegate":
                return k + 1
            outer = self._in_type
            self._scope(j + 1, k, walk_parent, enum_body=(self.java and kw == "enum"))
            self._in_type = outer
            return k + 1
        if chunk:
            self.chunks.append((ChunkType.CLASS, i, min(j, end - 1), name, None))
        return j + 1

    def _method(self, i: int, p: int, paren: int, end: int, parent: Optional[str]) -> int:
        t = self.t
        # name: the identifier before the parameter list (C#: before "<...>" type parameters)
        n = paren - 1
        if not self.java and n >= p and t[n].text == ">":
            depth = 0
            while n >= p:
                if t[n].text == ">":
                    depth += 1
                elif t[n].text == "<":
                    depth -= 1
                    if depth == 0:
                        n -= 1
                        break
                n -= 1
        operator = any(t[j].text == "operator" for j in range(p, paren))
        close = _match(t, paren)
        j = close + 1
        # throws / constructor initializer / constraints / default values up to the body or ';'
        while j < end and t[j].text not in ("{", ";", "=>"):
            j = _match(t, j) + 1 if t[j].text in ("(", "[") else j + 1
        if j < end and t[j].text == "{":
            last = _match(t, j)
        elif j < end and t[j].text == "=>":
            last = _until(t, j, end, (";",))
        else:
            last = min(j, end - 1)
        if operator or n < p or t[n].kind != "id":
            return last + 1
        if n > p and t[n - 1].text in (".", "~", "?."):
            return last + 1  # a call statement (C# top level) or a destructor: no chunk
        if n == p and parent is None:
            return last + 1  # a call statement: constructors exist only inside types
        if not self.java and not self._in_type:
            return last + 1  # C# top-level local function: no declaration node the reference chunks
        name = t[n].text
        self.decl_names.add(n)
        # tokens between the modifiers / type parameters and the name: the return type (none: constructor)
        q = p
        if self.java and q < n and t[q].text == "<":
            q = self._close_angle(q, n) + 1
        ret = list(range(q, n))
        if not self.java and len(ret) == 1 and t[ret[0]].kind == "id":
            name = t[ret[0]].text  # the first identifier child is the return type
        kind = ChunkType.METHOD if parent else ChunkType.FUNCTION
        self.chunks.append((kind, i, last, name, parent))
        return last + 1

    def _close_angle(self, i: int, end: int) -> int:
        depth = 0
        for j in range(i, end):
            x = self.t[j].text
            if x == "<":
                depth += 1
            elif x == ">":
                depth -= 1
                if depth == 0:
                    return j
            elif x == ">>":
                depth -= 2
                if depth <= 0:
                    return j
        return i

    def _field(self, i: int, p: int, end: int, parent: Optional[str]) -> int:
        t = self.t
        j = p
        assigned = False
        while j < end:
            x = t[j].text
            if x == ";":
                return j + 1
            if x in ("=", "=>"):
                assigned = True
            if x == "{":
                k = _match(t, j)
                if not assigned:
                    # a member with a block and no initializer: C# property / event
                    # accessors, a Java compact record constructor or initializer
                    return k + 1
                # Java anonymous class in an initializer: new X(...) { members }
                if self.java and j > 0 and t[j - 1].text == ")":
                    o = _match_back(t, j - 1)
                    if self._after_new(o):
                        outer = self._in_type
                        self._scope(j + 1, k, parent)
                        self._in_type = outer
                j = k + 1
                continue
            if x in ("(", "["):
                j = _match(t, j) + 1
                continue
            j += 1
        return end

    def _after_new(self, open_paren: int) -> bool:
        k = open_paren - 1
        while k >= 0 and self.t[k].text in (">", ".", "<") or (k >= 0 and self.t[k].kind == "id"):
            if self.t[k].text == "new":
                return True
            k -= 1
        return k >= 0 and self.t[k].text == "new"


def _chunks_from(toks: List[_Tok], scan: _Scanner, src: _Source) -> List[CodeChunk]:
    out = []
    for kind, a, b, name, parent in scan.chunks:
        b0, b1 = toks[a].b0, toks[b].b1
        line, eline = toks[a].line, toks[b].eline
        sig = line if kind in (ChunkType.CLASS, ChunkType.FUNCTION, ChunkType.METHOD) else None
        out.append(CodeChunk(kind, b0, b1, src.text(b0, b1), name, parent, line, eline, sig, sig))
    return out


_SCAN_CACHE: Dict[Tuple[str, str], Tuple[List[_Tok], _Scanner]] = {}


def _scan(code: str, lang: str) -> Tuple[List[_Tok], _Scanner]:
    """Tokens and declarations of a source (the segmenter and the analyser of
    one prompt share them; one entry kept)."""
    key = (code, lang)
    hit = _SCAN_CACHE.get(key)
    if hit is None:
        toks = _tokens(code, lang)
        sc = _Scanner(toks, lang)
        sc.scan()
        _SCAN_CACHE.clear()
        _SCAN_CACHE[key] = hit = (toks, sc)
    return hit


class BraceSegmenter:
    """Drop-in for ``TreeSitterSegmenter(tokenizer).segment_code(code,
    language)`` on Java and C# source (see the module docstring)."""

    def __init__(self, tokenizer=None):
        self.tokenizer = tokenizer

    def segment_code(self, code: str, language: Optional[str] = None) -> List[CodeChunk]:
        if not code or not code.strip():
            return []
        lang = _norm_language(language, code)
        if lang not in ("java", "c_sharp"):
            raise ValueError(f"BraceSegmenter handles Java and C# (got {lang})")
        src = _Source(code)
        toks, sc = _scan(code, lang)
        return PythonSegmenter._fill_gaps(src, _chunks_from(toks, sc, src))


class BraceReferenceAnalyzer:
    """Drop-in for ``CrossReferenceAnalyzer(chunks, code, language).analyze()``
    on Java and C# source (see the module docstring)."""

    def __init__(self, chunks, code: str, language: Optional[str] = None):
        self.chunks = chunks
        self.code = code
        self.language = _norm_language(language, code)
        self.chunk_by_name: Dict[str, List[int]] = {}
        self.chunk_by_line: Dict[int, int] = {}
        for i, c in enumerate(chunks):
            name = getattr(c, "name", "") or ""
            if name:
                self.chunk_by_name.setdefault(name, []).append(i)
            for ln in range(int(getattr(c, "start_line", 0) or 0), int(getattr(c, "end_line", 0) or 0) + 1):
                self.chunk_by_line[ln] = i
        self.references: List[Reference] = []

    def _add(self, line: int, name: Optional[str], kind: str) -> None:
        source = self.chunk_by_line.get(line)
        if source is None or not name:
            return
        for target in self.chunk_by_name.get(name, ()):
            if target != source:
                self.references.append(Reference(source, target, kind, name, line, 1.0))

    def analyze(self) -> List[Reference]:
        if self.language not in ("java", "c_sharp"):
            raise ValueError(f"BraceReferenceAnalyzer handles Java and C# (got {self.language})")
        toks, sc = _scan(self.code, self.language)
        java = self.language == "java"
        self.references = []
        t = toks
        not_calls = _JAVA_NOT_CALLS if java else _CS_NOT_CALLS

        def last_ident(a: int, b: int) -> Optional[str]:
            for k in range(b, a - 1, -1):
                if t[k].kind == "id" and not t[k].text.startswith("@"):
                    return t[k].text
            return None

        def chain_start(k: int) -> int:
            """First token of the postfix expression ending at token k."""
            while True:
                if k > 0 and t[k - 1].text in (".", "?."):
                    k -= 1
                    prev = k - 1
                    if prev < 0:
                        return k
                    if t[prev].text in (")", "]"):
                        k = _match_back(t, prev)
                        if k > 0 and (t[k - 1].kind == "id" or t[k - 1].text in ("this", "super", "base")):
                            k -= 1
                            if k > 0 and t[k - 1].text == "new":
                                k -= 1
                        continue
                    if t[prev].text == ">" and not java:
                        depth = 0
                        while prev >= 0:
                            if t[prev].text == ">":
                                depth += 1
                            elif t[prev].text == "<":
                                depth -= 1
                                if depth == 0:
                                    break
                            prev -= 1
                        k = max(prev - 1, 0)
                        continue
                    k = prev
                    continue
                return k

        def declared_here(name_tok: int, paren: int) -> bool:
            """``Type name(...) {`` inside a body (a method of a local or
            anonymous class, a C# local function) or a C# destructor
            ``~Name() {``: a declaration, no call."""
            if name_tok == 0:
                return False
            before = t[name_tok - 1]
            if not (before.kind == "id" or before.text in (">", "]", "void") or (before.text == "~" and not java) or
                    (before.kind == "kw" and before.text not in ("new", "return", "throw", "else", "case", "await"))):
                return False
            e = _match(t, paren)
            return e + 1 < n and t[e + 1].text in ("{", "throws", "=>")

        n = len(t)
        for k in range(n):
            x = t[k]
            if x.text == "new" and k + 1 < n:
                # object creation: new Type(args) [body]; arrays and anonymous objects are other nodes
                j = k + 1
                while j < n and (t[j].kind == "id" or t[j].text in (".", "<", ">", ",", ">>", "?")):
                    j += 1
                if j >= n or t[j].text != "(" or j == k + 1:
                    continue
                e = _match(t, j)
                if e + 1 < n and t[e + 1].text == "{" and java:
                    e = _match(t, e + 1)
                self._add(x.line, last_ident(k, e), "call")
                continue
            if x.text != "(" or k == 0:
                continue
            prev = k - 1
            if t[prev].kind == "id" and (t[prev].text.startswith("@") or declared_here(prev, k)):
                continue  # annotation arguments / a declaration
            if java:
                if t[prev].kind == "id" and prev not in sc.decl_names and t[prev].text not in not_calls:
                    if prev > 0 and t[prev - 1].text == "new":
                        continue
                    self._add(t[chain_start(prev)].line, t[prev].text, "call")
                elif t[prev].text in ("this", "super") and (prev == 0 or t[prev - 1].text in (";", "{", "}")):
                    self._add(t[prev].line, last_ident(prev, _match(t, k)), "call")
            else:
                callee_end = prev
                if t[prev].text == ">":
                    # generic method call Foo<T>(...): the type arguments belong to the callee
                    depth, q = 0, prev
                    while q >= 0:
                        if t[q].text == ">":
                            depth += 1
                        elif t[q].text == "<":
                            depth -= 1
                            if depth == 0:
                                break
                        q -= 1
                    if q <= 0 or t[q - 1].kind != "id":
                        continue
                    head = q - 1
                else:
                    head = prev
                if t[head].kind != "id" or head in sc.decl_names or t[head].text in not_calls:
                    continue
                if head > 0 and t[head - 1].text == "new":
                    continue
                start = chain_start(head)
                self._add(t[start].line, last_ident(start, callee_end), "call")
        # inheritance
        for first, hend, kind in sc.classes:
            hend = min(hend, n)  # a header cut off by the end of the file
            names: List[str] = []
            if kind == 0:  # Java class: extends (last identifier) + implements (every type identifier)
                j = first
                while j < hend:
                    if t[j].text == "extends":
                        e = _until(t, j + 1, hend, ("implements", "permits"))
                        nm = last_ident(j + 1, e - 1)
                        if nm:
                            names.append(nm)
                        j = e
                        continue
                    if t[j].text == "implements":
                        e = _until(t, j + 1, hend, ("permits",))
                        names.extend(t[q].text for q in range(j + 1, e) if t[q].kind == "id")
                        j = e
                        continue
                    j += 1
            elif kind == 1:  # C#: base list after ':' (up to "where" constraints)
                j = first
                while j < hend and t[j].text != ":":
                    if t[j].text in ("(", "["):
                        j = _match(t, j)
                    j += 1
                if j < hend:
                    e = _until(t, j + 1, hend, ("where",))
                    names.extend(t[q].text for q in range(j + 1, e) if t[q].kind == "id")
            for nm in names:
                self._add(t[first].line, nm, "inherit")
        return self.references


class StructureSegmenter:
    """Language-dispatching segmenter: Python through the ``ast`` rules of
    :mod:`sabrecoder_b200.structure`, Java and C# through this module."""

    def __init__(self, tokenizer=None):
        self.tokenizer = tokenizer

    def segment_code(self, code: str, language: Optional[str] = None) -> List[CodeChunk]:
        if not code or not code.strip():
            return []
        lang = _norm_language(language, code)
        if lang in ("java", "c_sharp"):
            return BraceSegmenter(self.tokenizer).segment_code(code, lang)
        return PythonSegmenter(self.tokenizer).segment_code(code, lang)


class StructureAnalyzer:
    """Language-dispatching analyser (see :class:`StructureSegmenter`)."""

    def __init__(self, chunks, code: str, language: Optional[str] = None):
        from .structure import PythonReferenceAnalyzer
        lang = _norm_language(language, code)
        impl = BraceReferenceAnalyzer if lang in ("java", "c_sharp") else PythonReferenceAnalyzer
        self._impl = impl(chunks, code, language=lang)
        self.references = self._impl.references

    def analyze(self):
        self.references = self._impl.analyze()
        return self.references
