"""CPU tests of the C ABI boundary (no GPU, no compute): the library loads,
exports every entry point include/gadeon_kv.h declares, and rejects bad
geometry before touching the device."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gadeon_kv.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gkv_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from gadeon_b200 import build, kv
    build.build()
    return kv.load_library()


def test_header_matches_binding():
    from gadeon_b200 import kv
    assert declared_symbols() == sorted(kv.EXPORTED)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", os.path.join(ROOT, "gadeon_b200", "libgadeonkv.so")],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (gkv_\w+)", out))
    assert set(declared_symbols()) <= exported


def test_version_and_error_string(lib):
    assert b"sm_100a" in lib.gkv_version()
    assert isinstance(lib.gkv_last_error(), bytes)


def test_header_compiles_as_c():
    src = "#include \"gadeon_kv.h\"\nint main(void){gkv_pool_config c={0};(void)c;return 0;}\n"
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.dirname(HEADER),
                        "-x", "c", "-", "-fsyntax-only"], input=src, text=True, capture_output=True)
    assert r.returncode == 0, r.stderr


@pytest.mark.parametrize("field,value,code", [
    ("head_dim", 96, 5),      # GKV_ERR_UNSUPPORTED
    ("page_tokens", 12, 1),   # not a power of two -> GKV_ERR_INVALID
    ("page_tokens", 32768, 1),
    ("kv_heads", 0, 1),
    ("num_pages", 0, 1),
])
def test_pool_create_rejects_geometry(lib, field, value, code):
    from gadeon_b200.kv import _PoolConfig
    cfg = _PoolConfig(0, 2, 256, 16, 64, 4, 64, 1)
    setattr(cfg, field, value)
    h = C.c_void_p()
    assert lib.gkv_pool_create(C.byref(cfg), C.byref(h)) == code
    assert not h.value
    assert len(lib.gkv_last_error()) > 0


def test_null_arguments(lib):
    assert lib.gkv_pool_create(None, None) == 1
    assert lib.gkv_seq_create(None, None) == 1
    assert lib.gkv_pool_destroy(None) == 0


def test_binding_refuses_bad_arguments_before_any_device_work(lib):
    """The Python layer's checks run before anything reaches the C ABI or a
    device: wrong shapes or dtypes, an m array of the wrong length, and
    pageable host tensors (a kernel could not reach them) are refused with
    GKV_ERR_INVALID -- here on a machine without a GPU."""
    import torch
    import gadeon_b200 as gk
    n, H, D, C = 2, 4, 8, 3
    s0 = torch.zeros((n, H, D, D), dtype=torch.float16)
    delta, k = torch.zeros((n, H, C, D)), torch.zeros((n, H, C, D))
    gcum = torch.zeros((n, H, C))
    proj, pre = torch.zeros((n, C, 16)), torch.zeros((n, 16, 3), dtype=torch.float16)
    bad = [
        lambda: gk.mtp_rollback([1, 2], s0, delta[:, :, :2], k, gcum),        # delta rows != C
        lambda: gk.mtp_rollback([1, 2], s0, delta, k.double(), gcum),         # k not fp32
        lambda: gk.mtp_rollback([1], s0, delta, k, gcum),                     # one m for two items
        lambda: gk.mtp_rollback([1, 2], s0, delta, k, gcum),                  # pageable host memory
        lambda: gk.gdn_rollback([1, 2], s0, delta, k, gcum, proj[:, :2], pre),  # proj rows != C
        lambda: gk.gdn_rollback([1, 2], s0.float(), delta, k, gcum, proj, pre),  # state fp32, conv tail fp16
        lambda: gk.conv_rollback([1, 2], proj, pre.float().double()),         # pre of no storage type
    ]
    for i, call in enumerate(bad):
        with pytest.raises(gk.GkvError) as e:
            call()
        assert e.value.code == gk.GKV_ERR_INVALID, i


def test_every_entry_point_cites_what_it_replaces():
    """Each block of declarations in the header carries the reference
    interface it replaces (file:line) or says that it has no counterpart."""
    assert not uncited_entry_points(open(HEADER).read())


def uncited_entry_points(text):
    """Declarations whose comment -- the one right above, or the previous
    declaration's when a group shares one -- names no reference location."""
    body = text[text.index("typedef struct gkv_pool gkv_pool;"):]
    cite = re.compile(r"\.(swift|metal):\d+|:\d+(-\d+)?\)|:\d+-\d+|counterpart", re.I)
    missing, comment, prev_end = [], "", 0
    for m in re.finditer(r"^(?:int|const char \*)\s*(gkv_\w+)\s*\(", body, re.M):
        between = body[prev_end:m.start()]
        if "/*" in between:
            comment = between[between.rindex("/*"):]
        if not cite.search(comment):
            missing.append(m.group(1))
        prev_end = body.index(";", m.end()) + 1
    return missing


def test_citation_check_catches_a_removed_citation():
    text = open(HEADER).read()
    assert uncited_entry_points(text.replace("Library version string.  No reference counterpart.",
                                             "Library version string.", 1)) == ["gkv_version"]
