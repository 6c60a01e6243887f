"""Host side of expert parallelism on CPU: the communicator id one rank makes
reaches every rank over torch.distributed (two gloo ranks), and the library's
argument checks refuse bad ids before NCCL is touched."""
import os

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import swiftlet_b200 as swl


def _rank(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, swl.ep_unique_id_broadcast(rank)))
    finally:
        dist.destroy_process_group()


def test_unique_id_reaches_every_rank():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert len(got[0]) == swl.EP_ID_BYTES and got[0] == got[1]


def test_unique_ids_differ():
    assert swl.ep_unique_id() != swl.ep_unique_id()


def test_short_id_buffer_is_refused():
    import ctypes as C
    buf = C.create_string_buffer(16)
    rc = swl.lib().swl_ep_unique_id(C.cast(buf, C.c_void_p), 16)
    assert rc == swl.SWL_ERR_INVALID


def _liveness_rank(rank: int, world: int, port: int, q) -> None:
    import datetime
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
    alive = swl.ep_store_liveness(store, rank, world, timeout_s=1.0)
    seen = [alive(0), alive(1)]  # both ranks take steps 0 and 1
    if rank == 0:
        seen.append(alive(2))   # rank 1 never enters step 2
    q.put((rank, seen))
    if rank == 0:
        import time
        time.sleep(0.5)


def test_store_liveness_reports_a_peer_that_stops():
    """The host side of the expert-parallel failure path on CPU: the
    heartbeat callback confirms every peer at each step and answers False
    (within its limit) when a peer stops entering steps."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_liveness_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == [True, True, False]
    assert got[1] == [True, True]
