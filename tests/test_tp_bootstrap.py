"""Host side of the tensor-parallel bootstrap on CPU: two gloo ranks exchange the
128-byte NCCL id made by rank 0 through libq35 and agree on it (no GPU involved)."""
import multiprocessing as mp
import os
import socket

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        from asicfortranai_b200.tp import exchange_unique_id
        uid = exchange_unique_id(dist)
        q.put((rank, uid))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent instead of a silent exit
        q.put((rank, repr(e)))


def test_unique_id_exchange_two_ranks():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert isinstance(got[0], bytes) and isinstance(got[1], bytes), got
    assert got[0] == got[1] and len(got[0]) == 128 and any(got[0])
