"""Code-structure chunk types.

Same members and fields as the reference's ``ChunkType`` / ``CodeChunk``
(methods/sabrecoder/semantic_chunker.py:21-44), so chunk lists produced by
the reference's segmenter can be passed to this library unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from typing import Optional


class ChunkType(Enum):
    IMPORT = "import"
    FUNCTION = "function"
    CLASS = "class"
    METHOD = "method"
    MODULE_CODE = "module_code"
    COMMENT = "comment"
    DOCSTRING = "docstring"


@dataclass
class CodeChunk:
    chunk_type: ChunkType
    start: int
    end: int
    text: str
    name: str = ""
    parent_name: Optional[str] = None
    start_line: int = 0
    end_line: int = 0
    signature_start_line: Optional[int] = None
    signature_end_line: Optional[int] = None


def type_name(ct) -> str:
    """Name of a chunk type given as this module's enum, the reference's enum
    (same member names) or a plain string."""
    return getattr(ct, "name", str(ct)).upper()


SIGNATURE_TYPES = {"FUNCTION", "CLASS", "METHOD"}


def chunks_from_spans(spanset) -> list:
    """CodeChunk list for a :class:`sabrecoder_b200.spans.SpanSet` (one token
    per line, so line = token + 1)."""
    tmap = {"import": ChunkType.IMPORT, "function": ChunkType.FUNCTION, "class": ChunkType.CLASS,
            "statement": ChunkType.MODULE_CODE}
    out = []
    for s in spanset.spans:
        sig = s.start + 1 if s.has_signature else None
        out.append(CodeChunk(tmap[s.tag], 0, 0, "", name=f"s{s.start}", start_line=s.start + 1,
                             end_line=s.end + 1, signature_start_line=sig, signature_end_line=sig))
    return out
