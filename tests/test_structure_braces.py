"""Java and C# code structure without tree-sitter (sabrecoder_b200.structure_braces).

Each expectation follows the reference's rules: chunk node types
(methods/sabrecoder/semantic_chunker.py:59-74), the pre-order walk that does
not enter function bodies (:172-214), names from the first identifier child
(:268-290), gap filling (:323-453); call and inheritance references
(methods/sabrecoder/reference_graph.py:87-157, :191-250). tree-sitter itself
is not installed, so these are restatements of those rules on the grammars'
documented node shapes (parity unpinned).
"""

import random

import pytest

import numpy as np

from sabrecoder_b200.structure_braces import StructureAnalyzer, StructureSegmenter

JAVA = """package com.example.app;

import java.util.List;
import static java.lang.Math.max;

/** Javadoc for the service. */
@Service
public class OrderService extends BaseService implements Runnable, Comparable<OrderService> {
    private final List<String> items = new ArrayList<>();
    private Runnable r = new Runnable() {
        @Override
        public void run() { helper(); }
    };

    public OrderService(int n) {
        super(n);
        this.items.add("x");
    }

    @Override
    public int compareTo(OrderService o) {
        return max(size(), o.size());
    }

    int size() { return items.size(); }

    static <T> T first(List<T> xs) {
        return xs.get(0);
    }

    interface Listener { void onEvent(String e); }

    enum Kind { A, B { void f() { } }; int code() { return 1; } }

    void helper() {
        Kind k = Kind.A;
        new Helper(k).go();
        first(items);
        Runnable q = new Runnable() { public void run() { } };
    }
}

class Helper {
    Helper(Object o) {}
    void go() {}
}
"""

CSHARP = """using System;
using System.Collections.Generic;

namespace Demo.App
{
    [Serializable]
    public class Repo : BaseRepo, IDisposable
    {
        private readonly List<int> _xs = new List<int>();
        public int Count { get; set; } = 0;

        public Repo(int n) : base(n) { Init(); }

        public Task Run() { return Task.CompletedTask; }

        public void Init() { var h = new Helper(_xs); h.Go<int>(); }

        public List<int> Items() => _xs;

        public void Dispose() { }

        ~Repo() { }

        public static Repo operator +(Repo a, Repo b) => a;
    }

    struct Point { public int X; public Point(int x) { X = x; } }

    interface IThing { void Do(); }

    class Derived : Repo, IThing { public void Do() { Init(); } }
}

Console.WriteLine("top level");
static void LocalTop() { }

class Helper { public Helper(object o) {} public void Go<T>() {} }
"""


def synthetic_source(lang: str, ncls: int = 30, nm: int = 3, seed: int = 0):
    """Seeded Java / C# file of ``ncls`` classes with ``nm`` methods each;
    every method body creates other classes and calls one of their methods.
    Returns the source and the reference set the rules give for it, as
    ``(source name, target name, kind)`` with chunk names."""
    r = random.Random(seed)
    java = lang == "java"
    out = ["package demo;", "import java.util.List;", ""] if java else ["using System;", "using System.Linq;", ""]
    names = [f"C{i}" for i in range(ncls)]
    refs = set()
    for i, c in enumerate(names):
        base = names[r.randrange(i)] if i and r.random() < 0.3 else None
        head = f"class {c}" + ((" extends " if java else " : ") + base if base else "") + " {"
        out.append(head)
        if base:
            # the class line is covered by the class chunk only
            refs.add((c, base, "inherit"))
        for m in range(nm):
            me = f"m{i}_{m}"
            out.append(f"    {'' if java else 'public '}int {me}(int x) {{")
            for _ in range(r.randrange(1, 3)):
                j, k = r.randrange(ncls), r.randrange(nm)
                out.append(f"        x += new {names[j]}().m{j}_{k}(x);")
                refs.add((me, names[j], "call"))            # creation: last identifier C<j>
                if f"m{j}_{k}" != me:
                    refs.add((me, f"m{j}_{k}", "call"))     # invocation: the method name
            out.append("        return x;")
            out.append("    }")
        out.append("}")
        out.append("")
    return "\n".join(out), refs


def _view(chunks):
    return [(c.chunk_type.name, c.name, c.parent_name, c.start_line, c.end_line) for c in chunks]


def test_java_chunks():
    ch = StructureSegmenter().segment_code(JAVA, "java")
    assert _view(ch) == [
        ("MODULE_CODE", "", None, 5, 6),               # blank line + Javadoc (comments are not part of nodes)
        ("IMPORT", "import", None, 1, 2),              # package_declaration; the blank line joins it
        ("IMPORT", "import", None, 3, 3),
        ("IMPORT", "import", None, 4, 4),
        ("CLASS", "OrderService", None, 7, 42),        # from its annotation to the closing brace
        ("METHOD", "run", "OrderService", 11, 12),     # anonymous class in a field initializer
        ("METHOD", "OrderService", "OrderService", 15, 18),  # constructor
        ("METHOD", "compareTo", "OrderService", 20, 23),
        ("METHOD", "size", "OrderService", 25, 25),
        ("METHOD", "first", "OrderService", 27, 29),   # generic method: the name, not the type T
        ("CLASS", "Listener", None, 31, 31),           # nested type: a CLASS chunk without parent
        ("METHOD", "onEvent", "Listener", 31, 31),
        ("CLASS", "Kind", None, 33, 33),               # enum_declaration is a class node in Java
        ("METHOD", "f", "Kind", 33, 33),               # method of an enum constant's body
        ("METHOD", "code", "Kind", 33, 33),
        ("METHOD", "helper", "OrderService", 35, 40),  # its body (and the class in it) is not walked
        ("CLASS", "Helper", None, 43, 47),
        ("METHOD", "Helper", "Helper", 44, 44),
        ("METHOD", "go", "Helper", 45, 45),
    ]
    assert ch[4].text.startswith("@Service\npublic class OrderService")
    assert ch[4].signature_start_line == 7 and ch[1].signature_start_line is None


def test_java_references():
    ch = StructureSegmenter().segment_code(JAVA, "java")
    refs = {(r.source_chunk_idx, r.target_chunk_idx, r.ref_type, r.name, r.line_number)
            for r in StructureAnalyzer(ch, JAVA, "java").analyze()}
    assert refs == {
        (4, 15, "call", "helper", 10),    # new Runnable() { ... helper(); }: the last identifier of the expression
        (5, 15, "call", "helper", 12),    # helper() inside run()
        (7, 8, "call", "size", 22),       # size() and o.size()
        (15, 18, "call", "go", 37),       # new Helper(k).go(): go; the creation names its last identifier, k
        (15, 9, "call", "first", 38),
        (15, 5, "call", "run", 39),       # new Runnable() { public void run() { } }: last identifier is run
        (4, 6, "inherit", "OrderService", 7),  # Comparable<OrderService>: every type identifier of implements
    }


def test_csharp_chunks():
    ch = StructureSegmenter().segment_code(CSHARP, "c_sharp")
    sem = [v for v in _view(ch) if v[0] != "MODULE_CODE"]
    assert sem == [
        ("IMPORT", "import", None, 1, 1),
        ("IMPORT", "import", None, 2, 2),              # lines 3-5 (namespace header) are a MODULE_CODE gap
        ("CLASS", "Repo", None, 6, 26),                # from its attribute list; the blank line 26 joins it
        ("METHOD", "Repo", "Repo", 12, 12),
        ("METHOD", "Task", "Repo", 14, 14),            # return type parsed as an identifier comes first
        ("METHOD", "Init", "Repo", 16, 16),
        ("METHOD", "Items", "Repo", 18, 18),           # expression-bodied
        ("METHOD", "Dispose", "Repo", 20, 20),         # destructor and operator: not chunks
        ("CLASS", "Point", None, 27, 28),              # struct_declaration
        ("METHOD", "Point", "Point", 27, 27),
        ("CLASS", "IThing", None, 29, 30),
        ("METHOD", "Do", "IThing", 29, 29),
        ("CLASS", "Derived", None, 31, 31),
        ("METHOD", "Do", "Derived", 31, 31),
        ("CLASS", "Helper", None, 37, 38),             # top-level statements and local functions: not chunks
        ("METHOD", "Helper", "Helper", 37, 37),
        ("METHOD", "Go", "Helper", 37, 37),
    ]
    gaps = [v[3:] for v in _view(ch) if v[0] == "MODULE_CODE"]
    assert gaps == [(3, 5), (32, 36)]


def test_csharp_references():
    ch = StructureSegmenter().segment_code(CSHARP, "c_sharp")
    names = [c.name for c in ch]
    refs = {(names[r.source_chunk_idx], names[r.target_chunk_idx], r.ref_type, r.name)
            for r in StructureAnalyzer(ch, CSHARP, "c_sharp").analyze()}
    assert ("Repo", "Init", "call", "Init") in refs        # constructor body
    assert ("Init", "Go", "call", "Go") in refs            # h.Go<int>(): int is no identifier
    assert ("Do", "Init", "call", "Init") in refs
    # class Derived : Repo, IThing { public void Do() ... } sits on one line; the later chunk
    # covering a line is the source of what starts there, so Do inherits
    assert ("Do", "Repo", "inherit", "Repo") in refs
    assert ("Do", "IThing", "inherit", "IThing") in refs
    assert ("Derived", "Repo", "inherit", "Repo") not in refs
    assert all(r[3] != "Repo" or r[2] != "call" for r in refs)  # ~Repo() { } is a declaration
    assert all(r[3] != "base" for r in refs)                     # ": base(n)" is no invocation
    # new Helper(_xs) names its last identifier, _xs: no chunk
    assert len(refs) == 5


def test_brackets_inside_literals_and_comments_do_not_count():
    java = ('''class A { String s = "}{ \\" {"; char c = '}'; char d = '\\''; /* { */ // }
  String t = """
     text { block "" } \\""" still
     """;
  void f() { g("a{", '{'); }
}
class B { void h() { f(); } }
''')
    ch = StructureSegmenter().segment_code(java, "java")
    assert [v for v in _view(ch) if v[0] != "MODULE_CODE"] == [
        ("CLASS", "A", None, 1, 6), ("METHOD", "f", "A", 5, 5), ("CLASS", "B", None, 7, 8), ("METHOD", "h", "B", 7, 7)]
    cs = ('''using System; // {
#region R {
class A { string s = @"verbatim "" {
 line2 }"; string r = """raw " {"" }"""; string i = $"x{y}z"; char c = '"';
  void F() { G("}", '\\\\'); }
#endregion
}
class B { void H() { F(); } }
''')
    ch = StructureSegmenter().segment_code(cs, "c_sharp")
    assert [v for v in _view(ch) if v[0] != "MODULE_CODE"] == [
        ("IMPORT", "import", None, 1, 1), ("CLASS", "A", None, 3, 7), ("METHOD", "F", "A", 5, 5),
        ("CLASS", "B", None, 8, 9), ("METHOD", "H", "B", 8, 8)]
    names = [c.name for c in ch]
    refs = {(names[r.source_chunk_idx], names[r.target_chunk_idx]) for r in StructureAnalyzer(ch, cs, "c_sharp").analyze()}
    assert refs == {("H", "F")}


def test_synthetic_sources_give_the_planted_references():
    for lang in ("java", "c_sharp"):
        code, want = synthetic_source(lang)
        ch = StructureSegmenter().segment_code(code, lang)
        assert sum(c.chunk_type.name == "CLASS" for c in ch) == 30
        assert sum(c.chunk_type.name == "METHOD" for c in ch) == 90
        names = [c.name for c in ch]
        got = {(names[r.source_chunk_idx], names[r.target_chunk_idx], r.ref_type)
               for r in StructureAnalyzer(ch, code, lang).analyze()}
        assert got == want


def test_builder_structure_for_java_without_tree_sitter():
    """The mask builder picks the built-in Java backend when tree-sitter is
    absent; its chunks, gap filling and dependency edges feed the oracle's
    block mask, which comes out causal with the class-level edges visible."""
    from oracle import mask_oracle as MO
    from sabrecoder_b200.sabrecoder_attention import StructureAwareMaskBuilder
    from sabrecoder_b200.spans import LineTokenizer
    mb = StructureAwareMaskBuilder(LineTokenizer(), block_size=4, window_size=4, num_prefix_tokens=0,
                                   num_suffix_tokens=0, global_last_k_chunks=0)
    seg, ana = mb._structure_backends()
    if seg is not StructureSegmenter:
        return  # the reference's tree-sitter modules are importable here
    st = mb._structure_for_code(JAVA, "java")
    ch = st["chunks"]
    assert {ch[i].name for i in st["import_chunks"]} == {"import"}
    assert len(st["import_chunks"]) == 3
    names = [c.name for c in ch]
    assert names.index("helper") in st["chunk_deps"][names.index("first")]
    L = len(JAVA.split("\n"))
    m = MO.build_block_mask_from_chunks(code=JAVA, seq_len=L, chunks=ch, chunk_deps=st["chunk_deps"],
                                       import_chunks=st["import_chunks"], language="java",
                                       tokenizer=LineTokenizer(), block_size=4, window_size=4,
                                       num_prefix_tokens=0, num_suffix_tokens=0, max_chunk_tokens=0,
                                       global_last_k_chunks=0)
    m = np.asarray(m).astype(bool)
    assert not np.triu(m, 1).any() and m.diagonal().all()
    assert m.sum() < np.tril(np.ones_like(m)).sum()  # sparse: some causal blocks are dropped


def test_language_detection_follows_the_reference_heuristic():
    """Without ``language`` the reference's marker order applies (C# markers
    first, methods/sabrecoder/semantic_chunker.py:104-125): a Java file with
    ``public class`` is scanned as C#; ``package`` alone marks Java."""
    from sabrecoder_b200.structure import detect_language
    assert detect_language(JAVA) == "c_sharp"
    java_only = "package p;\nclass A { void f() { } }\n"
    assert detect_language(java_only) == "java"
    assert _view(StructureSegmenter().segment_code(java_only)) == _view(StructureSegmenter().segment_code(java_only, "java"))
    assert _view(StructureSegmenter().segment_code(CSHARP)) == _view(StructureSegmenter().segment_code(CSHARP, "C#"))


JAVA_MORE = """package demo.more;

import java.util.*;
import java.util.function.Function;

@SuppressWarnings({"unchecked", "rawtypes"})
public final class Registry<K extends Comparable<K>, V> implements Iterable<Map.Entry<K, List<V>>> {
    private static final Map<String, Integer> CODES = new HashMap<>();
    static {
        CODES.put("a", 1);
    }
    private final Map<K, List<V>> map = new TreeMap<>((a, b) -> a.compareTo(b));

    public <R> List<R> mapAll(Function<? super V, ? extends R> fn) {
        List<R> out = new ArrayList<>();
        map.values().forEach(vs -> vs.forEach(v -> out.add(fn.apply(v))));
        return out;
    }

    @Override
    public Iterator<Map.Entry<K, List<V>>> iterator() { return map.entrySet().iterator(); }

    int kind(Object o) {
        return switch (o) {
            case Integer i when i > 0 -> 1;
            case String s -> { yield s.length(); }
            default -> 0;
        };
    }

    record Pair<A, B>(A first, B second) {
        Pair { Objects.requireNonNull(first); }
        static <T> Pair<T, T> twin(T t) { return new Pair<>(t, t); }
    }

    interface Visitor<T> {
        T visit(Object node);
        default T fallback() { return null; }
    }

    abstract static class Node {
        abstract int size();
        protected void touch() { mapAll(null); }
    }
}
"""

CSHARP_MORE = """using System;
using System.Collections.Generic;
using static System.Math;

namespace Demo.More;

[Obsolete("use V2", false)]
public sealed class Cache<TKey, TValue> : IDisposable where TKey : notnull
{
    private readonly Dictionary<TKey, TValue> _items = new();
    public event EventHandler? Changed;

    public int Count
    {
        get { return _items.Count; }
    }

    public TValue this[TKey key] => _items[key];

    public bool TryGet(TKey key, out TValue value) => _items.TryGetValue(key, out value);

    [Conditional("DEBUG")]
    public void Dump()
    {
        foreach (var (k, v) in _items) { Console.WriteLine($"{k}={v}"); }
        Changed?.Invoke(this, EventArgs.Empty);
    }

    public async System.Threading.Tasks.Task<int> LoadAsync() { await System.Threading.Tasks.Task.Yield(); return Max(1, 2); }

    public void Dispose() => _items.Clear();
}

public record Point(int X, int Y)
{
    public double Norm() => Sqrt(X * X + Y * Y);
}
"""


def _well_formed(code, chunks):
    n = len(code.split("\n"))
    for c in chunks:
        assert 1 <= c.start_line <= c.end_line <= n, (c.name, c.start_line, c.end_line, n)
    classes = {c.name: c for c in chunks if c.chunk_type.name == "CLASS"}
    for c in chunks:
        if c.chunk_type.name == "METHOD" and c.parent_name in classes:
            p = classes[c.parent_name]
            assert p.start_line <= c.start_line and c.end_line <= p.end_line, (c.name, c.parent_name)


def test_broader_java_syntax():
    ch = StructureSegmenter().segment_code(JAVA_MORE, "java")
    _well_formed(JAVA_MORE, ch)
    sem = [(c.chunk_type.name, c.name, c.parent_name) for c in ch if c.chunk_type.name != "MODULE_CODE"]
    names = [n for _, n, _ in sem]
    # generic methods, overrides and switch expressions are methods; the record's compact constructor and
    # static factory are walked with the outer class as parent (records are no chunks)
    for want in (("CLASS", "Registry", None), ("METHOD", "mapAll", "Registry"), ("METHOD", "iterator", "Registry"),
                 ("METHOD", "kind", "Registry"), ("METHOD", "twin", "Registry"), ("CLASS", "Visitor", None),
                 ("METHOD", "visit", "Visitor"), ("METHOD", "fallback", "Visitor"), ("CLASS", "Node", None),
                 ("METHOD", "size", "Node"), ("METHOD", "touch", "Node")):
        assert want in sem, (want, sem)
    assert "Pair" not in [n for k, n, _ in sem if k == "CLASS"]
    assert names.count("import") == 3
    refs = StructureAnalyzer(ch, JAVA_MORE, "java").analyze()
    by = {(ch[r.source_chunk_idx].name, ch[r.target_chunk_idx].name, r.ref_type) for r in refs}
    assert ("touch", "mapAll", "call") in by


def test_broader_csharp_syntax():
    ch = StructureSegmenter().segment_code(CSHARP_MORE, "c_sharp")
    _well_formed(CSHARP_MORE, ch)
    sem = [(c.chunk_type.name, c.name, c.parent_name) for c in ch if c.chunk_type.name != "MODULE_CODE"]
    for want in (("CLASS", "Cache", None), ("METHOD", "TryGet", "Cache"), ("METHOD", "Dump", "Cache"),
                 ("METHOD", "Dispose", "Cache")):
        assert want in sem, (want, sem)
    # properties, indexers and events are no methods; records are walked without being chunks
    assert not any(n in ("Count", "Changed", "this") for _, n, _ in sem)
    assert ("METHOD", "Norm", None) in sem or any(n == "Norm" for _, n, _ in sem)
    assert [n for _, n, _ in sem].count("import") == 3


@pytest.mark.parametrize("lang,code", [("java", JAVA), ("java", JAVA_MORE), ("c_sharp", CSHARP), ("c_sharp", CSHARP_MORE)])
def test_truncated_and_unbalanced_sources_do_not_fail(lang, code):
    rnd = random.Random(0)
    cuts = sorted({rnd.randrange(len(code)) for _ in range(25)}) + [len(code) // 2]
    for cut in cuts:
        for src in (code[:cut], code[:cut] + "}}}", "{{" + code[cut:], code.replace("}", "", 3)):
            ch = StructureSegmenter().segment_code(src, lang)
            _well_formed(src, ch)
            StructureAnalyzer(ch, src, lang).analyze()
