"""Multi-process host logic on CPU (gloo, world size 2): the rendezvous helpers that bench.py
and the tensor-parallel setup use — max-over-ranks device timing, the broadcast of the
128-byte NCCL unique id, and host-side failure detection (a rank that raises before a
collective makes the others fail with an error instead of waiting forever)."""
import importlib
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    sys.path.insert(0, ROOT)
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    vdist = importlib.import_module("webgpu-voxtral_b200.dist")
    try:
        assert vdist.init(backend="gloo", timeout_s=10.0)
        if mode == "ok":
            t = vdist.max_over_ranks(1.5 + rank)
            s = vdist.sum_over_ranks(10.0 * (rank + 1))
            uid = vdist.broadcast_bytes(bytes(range(128)) if rank == 0 else None)
            vdist.barrier()
            q.put((rank, t, s, uid))
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("injected host-side failure before the collective")
            vdist.max_over_ranks(1.0)   # rank 1 never joins: must end with an error, not hang
            q.put((rank, "no-error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", type(e).__name__))
    finally:
        try:
            vdist.shutdown()
        except Exception:  # noqa: BLE001
            pass


def _run(mode, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=timeout) for _ in range(world)]
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda x: x[0])


def test_max_sum_and_broadcast():
    out = _run("ok")
    for rank, t, s, uid in out:
        assert t == 2.5
        assert s == 30.0
        assert uid == bytes(range(128))


def test_failed_rank_surfaces_as_error():
    out = _run("fail", timeout=90)
    assert out[1][1] == "error"          # the injected failure
    assert out[0][1] == "error"          # the surviving rank's collective fails (timeout / closed peer)
