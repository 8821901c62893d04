"""bench.py's sharded probe on the CPU: two gloo ranks on 127.0.0.1 with the
device calls replaced by fakes that fail on one rank (at compile time, or in
the run as a rank whose peer's wait ran out would). Every rank must return,
agree that the sharded program cannot be used, and name why -- none may be
left waiting in a collective -- and with no failure both ranks agree to use
it."""
import datetime
import multiprocessing as mp
import os
import queue
import socket
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class _Buf:
    def __init__(self, n):
        self.ptr = 0x1000

    def upload(self, a):
        pass

    def free(self):
        pass


def _rank(rank, world, port, mode, q):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    import bench
    from cudacaml_b200 import backend_cuda as B
    from cudacaml_b200 import multi as M
    from cudacaml_b200 import runtime as R
    from cudacaml_b200.ir import F64, I32

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        class Prog:
            params = [("s0", F64, ()), ("vol", F64, ()), ("rate", F64, ()), ("seed", I32, ())]

        def compile_on(local, g, shard=None):
            if mode == "compile" and rank == 1:
                raise R.CcbError(4, "nvrtc said no")
            return Prog()

        class Peers:
            def __init__(self, c, exchange):
                exchange(b"h" * 64)  # the collective every rank takes part in
                if mode == "peers" and rank == 0:
                    raise R.CcbError(3, "cuIpcOpenMemHandle failed")

            def close(self):
                pass

        def run_device_ptrs(c, ins, outs, s):
            pass

        def check_device(c, s):
            if mode == "peers":  # the rank whose peer never ran: its bounded wait gave up
                raise R.CcbError(6, "cross-rank combine gave up")

        B.compile_on, B.run_device_ptrs, B.check_device, B.release = compile_on, run_device_ptrs, check_device, lambda c: None
        M.ShardPeers = Peers
        R.Buffer = _Buf

        def exchange(h):
            got = [None] * world
            dist.all_gather_object(got, h)
            return got

        q.put((rank, bench.sharded_probe(rank, world, 0, dist, exchange)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, ("error", repr(e))))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode", ["none", "compile", "peers"])
def test_sharded_probe_agreement(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.monotonic() + 120
    try:
        while len(got) < world and time.monotonic() < deadline:
            try:
                r, res = q.get(timeout=1)
            except queue.Empty:
                continue
            got[r] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert len(got) == world, got
    assert all(res[0] != "error" for res in got.values()), got
    oks = {res[0] for res in got.values()}
    assert oks == {mode == "none"}, got
    if mode != "none":
        assert all(res[1] for res in got.values()), got  # every rank says why
