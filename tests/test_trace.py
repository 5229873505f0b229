"""NVTX ranges around the library's entry points (the tracing counterpart of
the SDK's include/timing.h phase timers).  A small NVTX tool library
(tests/nvtx/nvtx_probe.c) is injected into a child process through
NVTX_INJECTION64_PATH; the child calls entry points with arguments they
refuse before any device work, so no GPU is needed, and the probe reports
which ranges were opened and that every one was closed."""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]

CHILD = r"""
import ctypes, sys
sys.path.insert(0, sys.argv[1])
import inference_c_b200 as P
lib = P.load()
e = ctypes.create_string_buffer(128)
lib.pkv_kv_append(None, None, None, None, None, 0, None, e, len(e))
lib.pkv_paged_decode(None, None, 0, None, ctypes.c_float(1.0), None, 3, 0, 0, None, 0, None,
                     e, len(e))
lib.pkv_paged_prefill(None, None, 0, None, None, 0, 0, ctypes.c_float(1.0), 1, None, 3, None,
                      e, len(e))
lib.pkv_sdpa_f16(None, None, None, None, None, 1, 8, 2, 4, 4, 128, ctypes.c_float(0.1), 1,
                 None, 0, None, e, len(e))
lib.pkv_step_begin(None, None, None, None, 0, None, e, len(e))
lib.pkv_step_end(None, 1, e, len(e))
lib.tensor_attention_decode_sequence_paged(None)
probe = ctypes.CDLL(sys.argv[2])
probe.probe_ranges.restype = ctypes.c_char_p
print(probe.probe_ranges().decode(), end="")
print("DEPTH", probe.probe_depth())
"""


def test_entry_points_open_and_close_nvtx_ranges(lib, tmp_path):
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("needs gcc to build the NVTX probe")
    from inference_c_b200 import _build
    probe = tmp_path / "libnvtx_probe.so"
    subprocess.run([cc, "-shared", "-fPIC", "-O1", "-I", str(_build.cuda_home() / "include"),
                    "-o", str(probe), str(ROOT / "tests" / "nvtx" / "nvtx_probe.c")],
                   check=True)
    env = dict(os.environ, NVTX_INJECTION64_PATH=str(probe))
    out = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(probe)], env=env,
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    lines = out.stdout.splitlines()
    assert lines[-1] == "DEPTH 0"
    assert lines[:-1] == ["pkv_kv_append", "pkv_paged_decode", "pkv_paged_prefill",
                          "pkv_sdpa_f16", "pkv_step_begin", "pkv_step_end",
                          "tensor_attention_decode_sequence_paged"]
