"""Host side of tensor parallelism on the CPU: two gloo ranks gather their
exchange-region handles with fyodor_b200.tp_exchange, which must return every
rank's handle in rank order (the order fyb_plan_tp_connect expects), and
reject a rank without a handle. fyodor_b200.tp_connect_all connects all
ranks or none: when one rank's plan creation or region opening fails, every
rank ends unconnected and its steps return -1 without launching (a stand-in
plan records whether a step would have launched)."""
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


class FakePlan:
    """Stands in for a shard plan on the CPU: connect/disconnect state and a
    step that returns -1 (no launch) unless connected, as plan_token does."""

    def __init__(self, rank, fail_connect):
        self.rank, self.fail_connect = rank, fail_connect
        self.connected, self.launches = False, 0

    def tp_handle(self):
        return bytes([self.rank + 1]) * 64

    def tp_connect(self, handles):
        if self.fail_connect:
            return -2
        assert [h[0] for h in handles] == list(range(1, len(handles) + 1))
        self.connected = True
        return 0

    def tp_disconnect(self):
        self.connected = False
        return 0

    def token(self, token, position):
        if not self.connected:
            return -1
        self.launches += 1
        return 0


def _connect_rank(rank, world, port, out_dir, failure):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    import fyodor_b200 as F
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        last = rank == world - 1
        plan = None if (failure == "create" and last) else FakePlan(rank, failure == "connect" and last)
        ok = F.tp_connect_all(plan)
        step = plan.token(1, 0) if plan is not None else -1
        launches = plan.launches if plan is not None else 0
        with open(os.path.join(out_dir, "c%d" % rank), "w") as f:
            f.write("%d %d %d" % (ok, step, launches))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("failure", ["none", "create", "connect"])
def test_connect_all_or_none(tmp_path, failure):
    import torch.multiprocessing as mp
    world = 3
    mp.spawn(_connect_rank, args=(world, _free_port(), str(tmp_path), failure), nprocs=world, join=True)
    for r in range(world):
        ok, step, launches = map(int, open(os.path.join(str(tmp_path), "c%d" % r)).read().split())
        if failure == "none":
            assert (ok, step, launches) == (1, 0, 1)
        else:
            assert (ok, step, launches) == (0, -1, 0)
