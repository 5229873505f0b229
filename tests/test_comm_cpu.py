"""Host logic of the NCCL all-gather with a deadline (pkv_comm_*), on the
CPU: NCCL is replaced by tests/fake_nccl/fake_nccl.c (loaded through
PKV_NCCL_LIBRARY), which simulates joining with files and records abort,
destroy and all-gather calls.  Covered: a communicator whose ranks all join;
two gloo ranks where the second never joins, so the first gives up at its
deadline, aborts the communicator and rolls its decode step back (the SDK's
transaction rollback, attention.c:159-166, on this repository's allocator);
and a collective whose stream never finishes (a stalled peer), which the
wait abandons at its deadline.  Each case runs in child processes because
the library loads NCCL once per process."""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys
import textwrap

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]

PRELUDE = textwrap.dedent(r"""
    import ctypes, os, sys, time
    sys.path.insert(0, os.environ["PKV_ROOT"])
    import inference_c_b200 as P
    lib = P.load()
    err = ctypes.create_string_buffer(512)

    def init(uid, nranks, rank, timeout):
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(uid, 256)
        t0 = time.monotonic()
        ok = lib.pkv_comm_init(buf, 256, nranks, rank, -1, ctypes.c_double(timeout),
                               ctypes.byref(h), err, len(err))
        return ok, h.value, time.monotonic() - t0

    def uid():
        buf = ctypes.create_string_buffer(256)
        assert lib.pkv_comm_unique_id(buf, 256, err, len(err)) == 1, err.value
        return buf.raw
""")


def _fake(tmp_path):
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("needs gcc")
    from inference_c_b200 import _build
    so = tmp_path / "libfake_nccl.so"
    subprocess.run([cc, "-shared", "-fPIC", "-O1", "-I", str(_build.cuda_home() / "include"),
                    "-o", str(so), str(ROOT / "tests" / "fake_nccl" / "fake_nccl.c")],
                   check=True)
    return so


def _env(tmp_path, so):
    return dict(os.environ, PKV_ROOT=str(ROOT), PKV_NCCL_LIBRARY=str(so),
                FAKE_NCCL_DIR=str(tmp_path), MASTER_ADDR="127.0.0.1")


def _run(code, env, timeout=120):
    out = subprocess.run([sys.executable, "-c", PRELUDE + textwrap.dedent(code)], env=env,
                         capture_output=True, text=True, timeout=timeout)
    assert out.returncode == 0, out.stdout + out.stderr
    return out.stdout


def test_all_ranks_join_and_collective_completes(lib, tmp_path):
    so = _fake(tmp_path)
    _run("""
        ok, h, _ = init(uid(), 1, 0, 5.0)
        assert ok == 1 and h, err.value
        send, recv = ctypes.create_string_buffer(64), ctypes.create_string_buffer(64)
        assert lib.pkv_comm_all_gather(h, send, recv, 64, None, ctypes.c_double(5.0), err,
                                       len(err)) == 1, err.value
        DONE = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p)(lambda a, s: 1)
        lib.pkv_internal_comm_set_probe(ctypes.c_void_p(h), DONE, None)
        assert lib.pkv_comm_wait(h, None, ctypes.c_double(5.0), err, len(err)) == 1, err.value
        assert lib.pkv_comm_aborted(h) == 0
        lib.pkv_comm_destroy(h)
    """, _env(tmp_path, so))
    log = (tmp_path / "log").read_text().splitlines()
    assert log == ["init nonblocking rank 0", "init blocking rank 0", "allgather rank 0",
                   "finalize rank 0", "finalize rank 0", "destroy rank 0", "destroy rank 0"]


WORKER = """
    import torch.distributed as dist
    rank = int(sys.argv[1])
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            init_method="tcp://127.0.0.1:" + os.environ["PORT"])
    box = [uid() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    joins = rank == 0 or os.environ["PEER_JOINS"] == "1"
    if rank == 0:
        # the SDK transaction on this repository's allocator: begin, length
        # check, reserve past + 1, then the collective; on failure roll back
        cache = P.PagedKVCache(16, 64, 4)
        seq = cache.sequence_create()
        assert cache.reserve(seq, 40) and cache.set_length(seq, 40)
        free0 = cache.free_blocks()
        assert cache.begin_decode(seq)
        assert cache.length(seq) == 40 and cache.reserve(seq, 49)
        ok, h, took = init(box[0], 2, 0, 1.0)
        if ok:
            assert cache.set_length(seq, 49)
        else:
            assert cache.set_length(seq, 40)  # rollback
        cache.end_decode(seq)
        print("RESULT", ok, round(took, 2), cache.length(seq), cache.free_blocks() == free0,
              err.value.decode())
        print("RELEASED", cache.release(seq))
        if ok:
            lib.pkv_comm_destroy(h)
    elif joins:
        ok, h, _ = init(box[0], 2, 1, 10.0)
        assert ok == 1, err.value
        lib.pkv_comm_destroy(h)
    dist.barrier()
    dist.destroy_process_group()
"""


@pytest.mark.parametrize("peer_joins", [True, False])
def test_gloo_ranks_peer_missing_rolls_the_step_back(lib, tmp_path, peer_joins):
    import socket
    so = _fake(tmp_path)
    with socket.socket() as s_:
        s_.bind(("127.0.0.1", 0))
        port = s_.getsockname()[1]
    env = dict(_env(tmp_path, so), PORT=str(port), PEER_JOINS="1" if peer_joins else "0")
    code = PRELUDE + textwrap.dedent(WORKER)
    procs = [subprocess.Popen([sys.executable, "-c", code, str(r)], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
             for r in (0, 1)]
    outs = [p.communicate(timeout=120) for p in procs]
    for p, (o, e) in zip(procs, outs):
        assert p.returncode == 0, o + e
    line = [x for x in outs[0][0].splitlines() if x.startswith("RESULT")][0].split(" ", 5)
    ok, took, length, same_free = int(line[1]), float(line[2]), int(line[3]), line[4]
    log = (tmp_path / "log").read_text()
    if peer_joins:
        assert ok == 1 and length == 49 and "abort" not in log
    else:
        # gave up at its 1 s deadline, aborted, and the step left no trace
        assert ok == 0 and 0.9 <= took < 10 and length == 40 and same_free == "True"
        assert "to join" in line[5] and "abort rank 0" in log
    assert "RELEASED 1" in outs[0][0]


def test_stalled_collective_is_abandoned_at_the_deadline(lib, tmp_path):
    so = _fake(tmp_path)
    out = _run("""
        ok, h, _ = init(uid(), 1, 0, 5.0)
        assert ok == 1, err.value
        send, recv = ctypes.create_string_buffer(64), ctypes.create_string_buffer(64)
        assert lib.pkv_comm_all_gather(h, send, recv, 64, None, ctypes.c_double(5.0), err,
                                       len(err)) == 1
        NEVER = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p)(lambda a, s: 0)
        lib.pkv_internal_comm_set_probe(ctypes.c_void_p(h), NEVER, None)
        t0 = time.monotonic()
        assert lib.pkv_comm_wait(h, None, ctypes.c_double(0.3), err, len(err)) == 0
        took = time.monotonic() - t0
        assert 0.25 <= took < 5, took
        assert b"did not finish" in err.value and lib.pkv_comm_aborted(h) == 1
        assert lib.pkv_comm_all_gather(h, send, recv, 64, None, ctypes.c_double(1.0), err,
                                       len(err)) == 0
        assert b"aborted" in err.value
        lib.pkv_comm_destroy(h)
        print("ok")
    """, _env(tmp_path, so))
    assert "ok" in out
    log = (tmp_path / "log").read_text().splitlines()
    # both communicators (the joining one and the collectives' one) aborted
    assert log.count("abort rank 0") == 2 and "destroy rank 0" not in log


def test_refuses_bad_arguments(lib):
    import ctypes
    err = ctypes.create_string_buffer(256)
    h = ctypes.c_void_p()
    assert lib.pkv_comm_init(None, 256, 2, 0, -1, ctypes.c_double(1.0), ctypes.byref(h), err,
                             len(err)) == 0
    assert lib.pkv_comm_unique_id(None, 256, err, len(err)) == 0
    assert lib.pkv_comm_wait(None, None, ctypes.c_double(1.0), err, len(err)) == 0
    assert lib.pkv_comm_aborted(None) == 1
