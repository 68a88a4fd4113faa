"""Row sharding across ranks: the host-side plan (CPU, gloo ranks) and the
library communicator (GPU: one rank, and a peer that never joins)."""
import ctypes as C
import os

import numpy as np
import pytest

from sharpinference_b200 import native

N = native


@pytest.mark.parametrize("rows", [1, 7, 3072, 5120, 200064, 100352])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_plan_covers_rows_once(rows, world):
    seen = np.zeros(rows, np.int32)
    pers = set()
    for r in range(world):
        b, c, per = native.rowshard_plan(rows, world, r)
        assert 0 <= c <= per and b + c <= rows
        seen[b:b + c] += 1
        pers.add(per)
    assert np.all(seen == 1) and len(pers) == 1


def test_plan_rejects_bad_arguments():
    with pytest.raises(native.ArgumentError):
        native.rowshard_plan(0, 2, 0)
    with pytest.raises(native.ArgumentError):
        native.rowshard_plan(10, 2, 2)


def _gloo_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        uid = [native.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ids = [None] * world
        dist.all_gather_object(ids, uid[0])
        plans = [None] * world
        dist.all_gather_object(plans, [native.rowshard_plan(n, world, rank) for n in (5120, 3072, 200064)])
        q.put((rank, len(set(ids)) == 1 and len(uid[0]) == 128, plans))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_share_id_and_partition_rows():
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    procs = [ctxm.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same_id, plans in results:
        assert same_id
        for shape_i, n in enumerate((5120, 3072, 200064)):
            covered = sum(plans[r][shape_i][1] for r in range(2))
            assert covered == n


@pytest.mark.gpu
def test_single_rank_comm_matches_plain_matvec(ctx):
    rows, cols = 5120, 3072
    blob = native.synth_weights(N.Q4_K, 3, rows, cols, 0.02)
    x = native.synth_normal(4, cols, 1.0)
    W, X, Y, R = ctx.buffer(blob.nbytes), ctx.buffer(cols * 4), ctx.buffer(rows * 4), ctx.buffer(rows * 4)
    comm = native.Comm(0, 1, 0, native.comm_unique_id(), timeout_ms=60000)
    try:
        W.upload(blob), X.upload(x)
        comm.rowshard_matvec_allgather(N.Q4_K, W.device_pointer, X.device_pointer, Y.device_pointer, rows, cols,
                                       ctx.stream)
        ctx.matvec(N.Q4_K, W, X, R, rows, cols)
        ctx.synchronize()
        assert np.array_equal(Y.readback().view(np.float32), R.readback().view(np.float32))
    finally:
        comm.close()
        for b in (W, X, Y, R):
            b.free()


@pytest.mark.gpu
def test_comm_create_times_out_when_peer_never_joins():
    """Failure detection on the host: rank 0 of 2 waits for a rank that never
    joins and gets SI_ERR_TIMEOUT after the deadline (nothing hangs)."""
    uid = (C.c_uint8 * 128).from_buffer_copy(native.comm_unique_id())
    h = C.c_void_p()
    st = native.lib.si_comm_create(0, 2, 0, uid, 3000, C.byref(h))
    assert st == N.SI_ERR_TIMEOUT, native.last_error()
    assert not h.value
