"""The Swift package (swift/): the reference's PagePool / hostFlashDecode
surface (leok7v/gadeon LLM/src/CoreML/PagedAttention.swift:21-366) over the C
ABI.  No Swift toolchain exists here, so these CPU tests check the package
against the header it binds: every gkv_* function and GKV_* constant the Swift
names is declared in include/gadeon_kv.h, every call passes as many arguments
as the declaration takes, the module map reaches the header and links the
library, and the wrapper carries the reference's method names and labels."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SWIFT = os.path.join(ROOT, "swift")
HEADER = os.path.join(ROOT, "include", "gadeon_kv.h")


def swift_sources():
    out = []
    for d, _, files in os.walk(SWIFT):
        out += [os.path.join(d, f) for f in files if f.endswith(".swift")]
    return out


def header_decls():
    """name -> number of parameters of every function the header declares."""
    text = open(HEADER).read()
    decls = {}
    for m in re.finditer(r"^(?:int|const char \*)\s*(gkv_\w+)\s*\(([^;]*?)\)\s*;", text, re.M | re.S):
        params = m.group(2).strip()
        decls[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return decls, text


def call_args(src, start):
    """Top-level arguments of the call whose '(' is at src[start]."""
    depth, args, cur = 0, [], ""
    for ch in src[start:]:
        if ch in "([{":
            depth += 1
            if depth == 1:
                continue
        elif ch in ")]}":
            depth -= 1
            if depth == 0:
                args.append(cur)
                break
        if depth == 1 and ch == ",":
            args.append(cur)
            cur = ""
        else:
            cur += ch
    return [a for a in args if a.strip()]


def test_swift_names_only_declared_symbols_with_their_arity():
    decls, text = header_decls()
    seen = set()
    for path in swift_sources():
        src = open(path).read()
        for m in re.finditer(r"\b(gkv_[a-z_0-9]+)\s*\(", src):
            name = m.group(1)
            if name == "gkv_pool_config":  # the struct's memberwise initializer (checked below)
                continue
            assert name in decls, f"{path}: {name} is not declared in gadeon_kv.h"
            n = len(call_args(src, m.end() - 1))
            assert n == decls[name], f"{path}: {name} called with {n} arguments, declared with {decls[name]}"
            seen.add(name)
        for c in set(re.findall(r"\bGKV_[A-Z_0-9]+\b", src)):
            assert re.search(rf"\b{c}\b", text), f"{path}: {c} is not in gadeon_kv.h"
    assert {"gkv_pool_create", "gkv_append", "gkv_seed", "gkv_truncate", "gkv_clone_seq", "gkv_compact_seq",
            "gkv_tile_at", "gkv_attend", "gkv_attend_ex", "gkv_append_attend_ex"} <= seen


def test_pool_config_fields_match_the_header():
    _, text = header_decls()
    fields = re.findall(r"^\s*(?:int32_t|uint64_t)\s+(\w+);", text[text.index("typedef struct gkv_pool_config"):
                                                              text.index("} gkv_pool_config;")], re.M)
    src = open(os.path.join(SWIFT, "Sources", "GadeonKV", "PagePool.swift")).read()
    m = re.search(r"gkv_pool_config\((.*?)\)\n", src, re.S)
    labels = re.findall(r"(\w+):", m.group(1))
    assert labels == fields, (labels, fields)


def test_module_map_reaches_the_header_and_links_the_library():
    d = os.path.join(SWIFT, "Sources", "CGadeonKV")
    mm = open(os.path.join(d, "module.modulemap")).read()
    assert re.search(r'link\s+"gadeonkv"', mm)
    shim = re.search(r'header\s+"([^"]+)"', mm).group(1)
    inc = re.search(r'#include\s+"([^"]+)"', open(os.path.join(d, shim)).read()).group(1)
    assert os.path.samefile(os.path.normpath(os.path.join(d, inc)), HEADER)
    pkg = open(os.path.join(SWIFT, "Package.swift")).read()
    assert '.systemLibrary(name: "CGadeonKV"' in pkg and 'dependencies: ["CGadeonKV"]' in pkg


def test_wrapper_carries_the_reference_api():
    """PagePool (PagedAttention.swift:21-287): init(P:kvHeads:dh:) :40,
    floats32() :46, pageCount :79, kPage/vPage :80-81, append(k:v:) :85,
    seed(K:V:count:) :99, tileAt(_:_:_:) :151, truncate(to:) :181,
    clone() :199, compact() :225, fromCompact(k:v:length:P:kvHeads:dh:) :256,
    length :27; hostFlashDecode(q:pool:G:) :317; pagedFlashBatched :376;
    Engine.verifyAttn (Engine.swift:2620)."""
    src = open(os.path.join(SWIFT, "Sources", "GadeonKV", "PagePool.swift")).read()
    for pat in [r"final class PagePool\b", r"init\(P: Int, kvHeads: Int, dh: Int\)", r"func floats32\(\)",
                r"var pageCount: Int", r"func kPage\(_ i: Int\)", r"func vPage\(_ i: Int\)",
                r"func append\(k: \[UInt16\], v: \[UInt16\]\) throws", r"func seed\(K: \[UInt16\], V: \[UInt16\], count: Int\) throws",
                r"func tileAt\(_ start: Int, _ count: Int, _ tileP: Int\) throws", r"func truncate\(to newLength: Int\)",
                r"func clone\(\) throws -> PagePool", r"func compact\(\) -> \(k: \[UInt16\], v: \[UInt16\]\)",
                r"static func fromCompact\(k: \[UInt16\], v: \[UInt16\], length: Int, P: Int, kvHeads: Int,\s*dh: Int\) throws -> PagePool",
                r"var length: Int", r"func hostFlashDecode\(q: \[UInt16\], pool: PagePool, G: Int\) -> \[Float\]",
                r"func pagedFlashBatched\(q: \[UInt16\], pool: PagePool, s0GlobalPos: Int, sCount: Int,",
                r"func verifyAttn\("]:
        assert re.search(pat, src), pat
