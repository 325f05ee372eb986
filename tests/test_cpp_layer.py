"""The header-only C++ layer (include/gadeon_kv.hpp, the Swift PagePool /
hostFlashDecode interface of LLM/src/CoreML/PagedAttention.swift:21-366 over
the C ABI).  CPU: the header compiles under -Wall -Wextra -Werror at C++11
and C++17, and tests/cpp/test_pagepool.cpp builds and links against the
product library and the oracle.  GPU: that program runs its oracle-checked
scenario (state bit-exact, attention within the path's tolerance, the
throwing paths) and must exit 0."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
INC = ["-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include")]
WARN = ["-Wall", "-Wextra", "-Werror"]


@pytest.mark.parametrize("std", ["c++11", "c++17"])
def test_header_compiles(std):
    src = ('#include "gadeon_kv.hpp"\nint main() { gadeon::check(GKV_OK);\n'
           '  void (*f)(int32_t, const int32_t *, int32_t, int32_t, int32_t, int32_t, const void *, const float *,\n'
           '            const float *, const float *, void *, int32_t, int32_t, const float *, const void *, void *,\n'
           '            cudaStream_t) = gadeon::rollbackGDN;\n'
           '  void (*g)(int32_t, const int32_t *, int32_t, int32_t, int32_t, int32_t, const float *, const float *,\n'
           '            const float *, const float *, float *, int32_t, int32_t, const float *, const float *, float *,\n'
           '            cudaStream_t) = gadeon::rollbackGDN;\n'
           '  return f && g ? 0 : 1; }\n')
    r = subprocess.run(["g++", f"-std={std}", *WARN, *INC, "-x", "c++", "-", "-fsyntax-only"],
                       input=src, text=True, capture_output=True)
    assert r.returncode == 0, r.stderr


def test_half_to_float_exhaustive(tmp_path):
    """gadeon::detail::half_to_float (the widening of floats32()) equals
    numpy's binary16 -> binary32 for all 65,536 bit patterns."""
    import numpy as np
    src = tmp_path / "h2f.cpp"
    src.write_text('#include "gadeon_kv.hpp"\n#include <cstdio>\n'
                   'int main() { for (unsigned h = 0; h < 65536; ++h) { float f = gadeon::detail::half_to_float('
                   '(uint16_t)h); uint32_t b; std::memcpy(&b, &f, 4); std::printf("%u\\n", b); } return 0; }\n')
    exe = str(tmp_path / "h2f")
    r = subprocess.run(["g++", "-std=c++17", "-O1", *WARN, *INC, str(src), "-o", exe], text=True, capture_output=True)
    assert r.returncode == 0, r.stderr
    got = np.array(subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split(), dtype=np.uint64)
    want = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32).view(np.uint32)
    assert np.array_equal(got.astype(np.uint32), want)


def build_test_program(out_dir):
    from gadeon_b200 import build
    build.build()
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
    exe = os.path.join(out_dir, "test_pagepool")
    libdirs = [os.path.join(ROOT, "gadeon_b200"), os.path.join(ROOT, "oracle"), os.path.join(CUDA, "lib64")]
    cmd = ["g++", "-std=c++17", "-O1", *WARN, *INC, os.path.join(ROOT, "tests", "cpp", "test_pagepool.cpp"),
           "-o", exe, "-L", libdirs[0], "-lgadeonkv", "-L", libdirs[1], "-loracle", "-L", libdirs[2], "-lcudart",
           "-Wl,-rpath," + ":".join(libdirs)]
    r = subprocess.run(cmd, text=True, capture_output=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_program_builds(tmp_path):
    exe = build_test_program(str(tmp_path))
    assert os.access(exe, os.X_OK)


@pytest.mark.gpu
def test_program_passes_on_gpu(tmp_path):
    exe = build_test_program(str(tmp_path))
    r = subprocess.run([exe], text=True, capture_output=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all checks passed" in r.stdout
