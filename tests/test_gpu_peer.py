"""The peer-store all-gather (pkv_peer_*): every rank stores its bytes into
every rank's area over NVLink and waits, bounded, for the others' bytes.
On one GPU: a single-rank gather returns its input on repeated calls; a
two-rank gather whose second rank never stores (its area simulated by a
local buffer nobody writes) gives up at its deadline with fault code 4,
leaves the output untouched and the GPU usable.  With two or more GPUs: two
processes gather step-dependent data through each other's memory."""
from __future__ import annotations

import ctypes
import os
import pathlib
import socket
import subprocess
import sys
import textwrap

import pytest

import inference_c_b200 as P

pytestmark = pytest.mark.gpu
ROOT = pathlib.Path(__file__).resolve().parents[1]


def test_single_rank_gathers_its_input(lib, cuda):
    import torch
    g = P.PeerGather(0, 1, 0, 2048)
    try:
        g.connect([g.ipc_handle])
        for step in range(3):
            send = torch.arange(1024, device=cuda, dtype=torch.float16) + step
            recv = torch.full((1024,), float("nan"), device=cuda, dtype=torch.float16)
            g.all_gather(send, recv)
            torch.cuda.synchronize()
            assert torch.equal(recv, send)
    finally:
        g.destroy()
    assert P.device_fault(0) == 0


def test_missing_peer_gives_up_at_the_deadline(lib, cuda):
    import torch
    g = P.PeerGather(0, 2, 0, 2048)
    try:
        area_bytes = lib.pkv_internal_peer_gather_area_bytes
        area_bytes.restype, area_bytes.argtypes = ctypes.c_size_t, [ctypes.c_void_p]
        fake = torch.zeros(area_bytes(ctypes.c_void_p(g.handle)), dtype=torch.uint8, device=cuda)
        set_area = lib.pkv_internal_peer_gather_set_area
        set_area.restype = ctypes.c_int
        set_area.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        assert set_area(ctypes.c_void_p(g.handle), 1, ctypes.c_void_p(fake.data_ptr())) == 1
        send = torch.ones(1024, device=cuda, dtype=torch.float16)
        recv = torch.full((2048,), 7.0, device=cuda, dtype=torch.float16)
        g.all_gather(send, recv, timeout_s=0.2)  # rank 1's flag never comes
        torch.cuda.synchronize()
        assert P.device_fault(0) == 4
        assert torch.all(recv == 7.0)
        # our slot of step 1 (parity 1) reached "rank 1": area offset (1 * 2 + 0) * 2048
        assert torch.equal(fake[4096:6144], send.view(torch.uint8))
    finally:
        g.destroy()
    test_single_rank_gathers_its_input(lib, cuda)  # the GPU is still usable


CHILD = textwrap.dedent(r"""
    import os, sys, torch, torch.distributed as dist
    sys.path.insert(0, sys.argv[1])
    import inference_c_b200 as P
    rank = int(sys.argv[2])
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            init_method="tcp://127.0.0.1:" + sys.argv[3])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    g = P.PeerGather(rank, 2, rank, 4096)
    handles = [None, None]
    dist.all_gather_object(handles, g.ipc_handle)
    g.connect(handles)
    for step in range(5):
        send = torch.arange(2048, device=dev, dtype=torch.float16) * 0 + (10 * rank + step)
        recv = torch.empty(4096, device=dev, dtype=torch.float16)
        g.all_gather(send, recv, timeout_s=5.0)
        torch.cuda.synchronize()
        want = torch.cat([torch.full((2048,), 10 * r + step, dtype=torch.float16)
                          for r in range(2)]).to(dev)
        assert torch.equal(recv, want), (rank, step)
    assert P.device_fault(rank) == 0
    dist.barrier()
    g.destroy()
    dist.barrier()
    dist.destroy_process_group()
    print("ok", rank)
""")


def test_two_gpus_gather_each_others_bytes(lib, cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s_:
        s_.bind(("127.0.0.1", 0))
        port = str(s_.getsockname()[1])
    env = dict(os.environ, MASTER_ADDR="127.0.0.1")
    procs = [subprocess.Popen([sys.executable, "-c", CHILD, str(ROOT), str(r), port], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
             for r in (0, 1)]
    outs = [p.communicate(timeout=180) for p in procs]
    for p, (o, e) in zip(procs, outs):
        assert p.returncode == 0, o + e
