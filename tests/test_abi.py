"""The C ABI boundary, checked without a GPU: the library loads, exports every
function include/*.h declares (and the Python view binds them all), rejects
bad arguments with a 0 result and a message before touching the device, and
neither links nor names the oracle."""
from __future__ import annotations

import ctypes
import pathlib
import re
import subprocess

import pytest

import inference_c_b200 as P

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _declared_functions() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"^typedef[^;]*;", "", text, flags=re.M | re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(\w+)\s*\(", text, flags=re.M):
            name = m.group(1)
            if name not in {"if", "return", "typedef", "sizeof"}:
                names.add(name)
    return names


def test_every_declared_symbol_is_exported(lib):
    declared = _declared_functions()
    assert len(declared) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", str(P.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = declared - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    assert declared <= set(P.EXPORTS), sorted(declared - set(P.EXPORTS))


def test_product_does_not_link_or_name_the_oracle(lib):
    out = subprocess.run(["nm", "-D", str(P.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    assert "orc_" not in out and "ref_job" not in out
    needed = subprocess.run(["readelf", "-d", str(P.LIB_PATH)], capture_output=True, text=True,
                            check=True).stdout
    assert "oracle" not in needed
    for f in (ROOT / "inference_c_b200").rglob("*"):
        if f.suffix in {".py", ".c", ".cu", ".cuh", ".h"}:
            assert "oracle" not in f.read_text().replace("oracle-free", ""), f


def test_sm100a_only(lib):
    """Kernels are built for sm_100a and nothing else."""
    out = subprocess.run(["cuobjdump", "--list-elf", str(P.LIB_PATH)], capture_output=True,
                         text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    arches = set(re.findall(r"sm_\w+", out.stdout))
    assert arches == {"sm_100a"}, arches


def _err():
    return ctypes.create_string_buffer(256)


def test_kernel_entry_points_reject_bad_arguments(lib):
    e = _err()
    assert lib.pkv_kv_append(None, None, None, None, None, 0, None, e, len(e)) == 0
    assert b"null" in e.value
    layer = P.PkvPagedLayer(16, 16, 16, 4, 2, 128, 7)  # bad dtype
    batch = P.PkvBatch(16, 4, 16, 1)
    e = _err()
    assert lib.pkv_kv_append(ctypes.byref(layer), ctypes.byref(batch), None, 16, 16, 1, None, e,
                             len(e)) == 0
    assert b"dtype" in e.value
    layer.dtype = P.PKV_DTYPE_F16
    e = _err()
    assert lib.pkv_kv_append(ctypes.byref(layer), ctypes.byref(batch), None, 16, 16, 2, None, e,
                             len(e)) == 0  # one row per sequence needs total_rows == batch
    assert b"total_rows" in e.value
    e = _err()
    assert lib.pkv_kv_append(ctypes.byref(layer), ctypes.byref(batch), None, 24, 16, 1, None, e,
                             len(e)) == 0
    assert b"aligned" in e.value
    # decode: GQA group 3 and head_dim 96 are rejected up front
    e = _err()
    assert lib.pkv_paged_decode(ctypes.byref(layer), ctypes.byref(batch), 6, 16,
                                ctypes.c_float(0.1), 16, P.PKV_DTYPE_F32, 64, 0, 256, 1 << 20,
                                None, e, len(e)) == 0
    assert b"q_heads/kv_heads" in e.value
    layer.head_dim = 96
    e = _err()
    assert lib.pkv_paged_decode(ctypes.byref(layer), ctypes.byref(batch), 4, 16,
                                ctypes.c_float(0.1), 16, P.PKV_DTYPE_F32, 64, 0, 256, 1 << 20,
                                None, e, len(e)) == 0
    assert b"head_dim" in e.value
    layer.head_dim = 128
    e = _err()
    assert lib.pkv_paged_decode(ctypes.byref(layer), ctypes.byref(batch), 4, 16,
                                ctypes.c_float(float("nan")), 16, P.PKV_DTYPE_F32, 64, 0, 256,
                                1 << 20, None, e, len(e)) == 0
    e = _err()
    assert lib.pkv_paged_decode(ctypes.byref(layer), ctypes.byref(batch), 4, 16,
                                ctypes.c_float(0.1), 16, P.PKV_DTYPE_F32, 64, 0, 256, 8, None, e,
                                len(e)) == 0
    assert b"workspace" in e.value
    # decode with the append: the rows are checked first, then everything
    # pkv_paged_decode checks, before any device work
    e = _err()
    assert lib.pkv_paged_decode_append(ctypes.byref(layer), ctypes.byref(batch), None, 16, 4, 16,
                                       ctypes.c_float(0.1), 16, P.PKV_DTYPE_F32, 64, 0, 256,
                                       1 << 20, None, e, len(e)) == 0
    assert b"null key_rows" in e.value
    e = _err()
    assert lib.pkv_paged_decode_append(ctypes.byref(layer), ctypes.byref(batch), 16, 24, 4, 16,
                                       ctypes.c_float(0.1), 16, P.PKV_DTYPE_F32, 64, 0, 256,
                                       1 << 20, None, e, len(e)) == 0
    assert b"16-byte aligned" in e.value
    e = _err()
    assert lib.pkv_paged_decode_append(ctypes.byref(layer), ctypes.byref(batch), 16, 16, 6, 16,
                                       ctypes.c_float(0.1), 16, P.PKV_DTYPE_F32, 64, 0, 256,
                                       1 << 20, None, e, len(e)) == 0
    assert b"q_heads/kv_heads" in e.value and b"pkv_paged_decode_append" in e.value
    e = _err()
    assert lib.pkv_paged_decode_append(ctypes.byref(layer), ctypes.byref(batch), 16, 16, 4, 16,
                                       ctypes.c_float(0.1), 16, P.PKV_DTYPE_F32, 64, 0, 256, 8,
                                       None, e, len(e)) == 0
    assert b"workspace" in e.value
    e = _err()
    assert lib.pkv_step_begin(None, None, None, None, 0, None, e, len(e)) == 0
    assert lib.pkv_step_end(None, 1, e, len(e)) == 0


def test_dense_and_selftest_entry_points_reject_bad_arguments(lib):
    """Validation that happens before any device work (no GPU needed)."""
    f = ctypes.c_float
    e = _err()
    assert lib.pkv_sdpa_f16(None, None, None, None, None, 1, 8, 2, 4, 4, 128, f(0.1), 1,
                            None, 0, None, e, len(e)) == 0
    assert b"null" in e.value
    e = _err()  # q_heads not a multiple of kv_heads
    assert lib.pkv_sdpa_f16(16, 16, 16, None, 16, 1, 6, 4, 4, 4, 128, f(0.1), 1, 256,
                            1 << 20, None, e, len(e)) == 0
    assert b"multiple" in e.value
    e = _err()  # non-finite scale
    assert lib.pkv_sdpa_f16(16, 16, 16, None, 16, 1, 8, 2, 4, 4, 128, f(float("inf")), 1,
                            256, 1 << 20, None, e, len(e)) == 0
    assert b"finite" in e.value
    e = _err()  # causal must be 0 or 1
    assert lib.pkv_sdpa_f16(16, 16, 16, None, 16, 1, 8, 2, 4, 4, 128, f(0.1), 2, 256,
                            1 << 20, None, e, len(e)) == 0
    e = _err()  # head_dim must be 64 or 128
    assert lib.pkv_sdpa_f16(16, 16, 16, None, 16, 1, 8, 2, 4, 4, 96, f(0.1), 1, 256,
                            1 << 20, None, e, len(e)) == 0
    assert b"head_dim" in e.value
    e = _err()  # workspace too small
    assert lib.pkv_sdpa_f16(16, 16, 16, None, 16, 1, 8, 2, 4, 4, 64, f(0.1), 1, 256, 8,
                            None, e, len(e)) == 0
    assert b"workspace" in e.value
    # the host hook refuses head_dim other than 64 / 128 and value_dim != head_dim
    assert lib.pkv_sdpa_f16_host(16, 16, 16, None, 16, 1, 8, 2, 4, 4, 96, 96, f(0.1), 1) == 0
    assert lib.pkv_sdpa_f16_host(16, 16, 16, None, 16, 1, 8, 2, 4, 4, 128, 64, f(0.1), 1) == 0
    e = _err()
    assert lib.pkv_selftest_wait_timeout(None, e, len(e)) == 0
    assert b"null" in e.value


def test_workspace_size_is_monotonic(lib):
    small = lib.pkv_decode_workspace_bytes(1, 8, 64, 512, 0)
    big = lib.pkv_decode_workspace_bytes(32, 32, 128, 4096, 0)
    bigger = lib.pkv_decode_workspace_bytes(256, 32, 128, 32768, 0)
    assert 0 < small <= big < bigger
    assert bigger % 256 == 0
    # the tensor-core layout keeps its tickets and claim words at fixed offsets
    # and sizes its partials by work units, not by batch
    assert lib.pkv_decode_workspace_bytes(1, 32, 128, 4096, 0) == big


def test_python_view_fails_loudly_without_library(monkeypatch, tmp_path):
    monkeypatch.setattr(P, "LIB_PATH", tmp_path / "missing.so")
    monkeypatch.setattr(P, "_lib", None)
    with pytest.raises(RuntimeError, match="no fallback"):
        P.load()
