"""Host side of tensor parallelism on the CPU: two gloo ranks gather their
exchange-region handles with fyodor_b200.tp_exchange, which must return every
rank's handle in rank order (the order fyb_plan_tp_connect expects), and
reject a rank without a handle."""
import os
import socket

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir, bad):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    import fyodor_b200 as F
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        handle = bytes([rank + 1]) * F.IPC_HANDLE_BYTES
        if bad and rank == world - 1:
            handle = b"short"
        try:
            got = F.tp_exchange(handle)
            result = b"".join(got)
        except ValueError:
            result = b"rejected"
        with open(os.path.join(out_dir, "r%d" % rank), "wb") as f:
            f.write(result)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bad", [False, True])
def test_handle_exchange_order(tmp_path, bad):
    import torch.multiprocessing as mp

    import fyodor_b200 as F
    world = 2
    mp.spawn(_rank, args=(world, _free_port(), str(tmp_path), bad), nprocs=world, join=True)
    for r in range(world):
        data = open(os.path.join(str(tmp_path), "r%d" % r), "rb").read()
        if bad:
            assert data == b"rejected"
        else:
            assert data == b"".join(bytes([j + 1]) * F.IPC_HANDLE_BYTES for j in range(world))
