"""The C11 allocator (inference_c_b200/csrc/paged_kv_cache.c) under the
compilers' sanitizers, on the CPU: a threaded stress program
(tests/sanitize/alloc_stress.c: eight threads, an ownership check on every
page, a release hook that re-enters the cache) under AddressSanitizer +
UndefinedBehaviorSanitizer and under ThreadSanitizer, and the SDK's own
allocator unit test under ASan + UBSan where the SDK's sources are present.
Any report fails the run (-fno-sanitize-recover, halt_on_error)."""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
ALLOC = ROOT / "inference_c_b200" / "csrc" / "paged_kv_cache.c"
INC = ["-I", str(ROOT / "include"), "-I", str(ROOT / "inference_c_b200" / "csrc")]
SANITIZERS = {
    "asan_ubsan": ["-fsanitize=address,undefined", "-fno-omit-frame-pointer",
                   "-fno-sanitize-recover=all"],
    "tsan": ["-fsanitize=thread"],
}
ENV = dict(os.environ, ASAN_OPTIONS="halt_on_error=1:detect_leaks=1",
           UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1",
           TSAN_OPTIONS="halt_on_error=1:second_deadlock_stack=1")


def _build(tmp_path, name, sources, flags, extra=()):
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("needs gcc")
    exe = tmp_path / name
    subprocess.run([cc, "-std=gnu11", "-O1", "-g", "-UNDEBUG", *flags, *INC, *extra, "-o",
                    str(exe), *map(str, sources), "-lpthread"], check=True)
    return exe


@pytest.mark.parametrize("kind", sorted(SANITIZERS))
def test_allocator_stress_under_sanitizer(tmp_path, kind):
    exe = _build(tmp_path, f"stress_{kind}", [ROOT / "tests" / "sanitize" / "alloc_stress.c",
                                              ALLOC], SANITIZERS[kind])
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300, env=ENV)
    assert out.returncode == 0, out.stderr[-4000:]
    assert "stress ok" in out.stdout
    assert "Sanitizer" not in out.stderr, out.stderr[-4000:]


def test_sdk_allocator_test_under_asan_ubsan(tmp_path):
    ref = pathlib.Path(os.environ.get("REF", ROOT.parent / "reference"))
    src = ref / "tests" / "test_paged_kv_cache.c"
    if not src.exists():
        pytest.skip("needs the SDK's test source")
    exe = _build(tmp_path, "sdk_alloc_asan", [src, ALLOC], SANITIZERS["asan_ubsan"])
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120, env=ENV)
    assert out.returncode == 0, out.stderr[-4000:]
    assert "allocator tests passed" in out.stdout
