"""Row-sharded GEMV with the output exchange fused into the kernel
(si_rowshard_matvec_peer): one rank on one GPU, a peer that never arrives
(bounded wait, error bit, usable context afterwards), and two ranks on two
GPUs (skipped on one GPU)."""
import os
import socket

import numpy as np
import pytest

import oracle
from helpers import north_star_gate, row_norm_max
from sharpinference_b200 import native

pytestmark = pytest.mark.gpu
N = native
ARENA = 8 << 20
ERR_PEER_TIMEOUT = 16


def _case(wt, rows, cols, seed):
    blob = N.synth_weights(wt, seed, rows, cols, 0.02)
    x = N.synth_normal(seed + 50, cols, 1.0)
    return blob, x, oracle.matvec(wt, blob, x, rows, cols)


@pytest.mark.parametrize("wt,rows,cols", [(N.Q4_K, 5120, 3072), (N.Q8_0, 3000, 5120), (N.Q4_K, 3072, 8192)])
def test_single_rank_group_matches_oracle_and_replays(ctx, wt, rows, cols):
    blob, x, ref = _case(wt, rows, cols, 3)
    W, X, A = ctx.buffer(blob.nbytes), ctx.buffer(4 * cols), ctx.buffer(ARENA)
    W.upload(blob), X.upload(x)
    g = N.PeerGroup(0, 1, 0, [A.device_pointer], ARENA)
    try:
        offs = [0, 1 << 20]  # consecutive calls alternate output offsets
        for i in range(4):
            g.rowshard_matvec(wt, W.device_pointer, X.device_pointer, offs[i % 2], rows, cols, ctx.stream)
        ctx.synchronize()
        for off in offs:
            y = A.readback(4 * rows, offset=off).view(np.float32)
            north_star_gate(y, ref, x, row_norm_max(wt, blob, rows, cols), cols)
        graph = ctx.record(lambda: [g.rowshard_matvec(wt, W.device_pointer, X.device_pointer, offs[i % 2], rows,
                                                      cols, ctx.stream) for i in range(6)])
        for _ in range(3):
            graph.launch()
        ctx.synchronize()
        graph.close()
        y = A.readback(4 * rows, offset=offs[1]).view(np.float32)
        north_star_gate(y, ref, x, row_norm_max(wt, blob, rows, cols), cols)
        assert N.device_error_take(0) == 0
    finally:
        g.close()
        W.free(), X.free(), A.free()


def test_peer_that_never_arrives_times_out_and_context_survives(ctx):
    """Rank 0 of a 2-rank group whose 'peer' arena is a second local buffer
    that nobody drives: its flag never arrives, the kernel's bounded wait
    (2 s) gives up, sets the device error bit and the kernel completes."""
    rows, cols = 1024, 3072
    blob, x, ref = _case(N.Q4_K, rows, cols, 5)
    W, X = ctx.buffer(blob.nbytes), ctx.buffer(4 * cols)
    A0, A1 = ctx.buffer(ARENA), ctx.buffer(ARENA)
    W.upload(blob[: blob.nbytes // 2]), X.upload(x)
    A1.upload(np.zeros(ARENA, np.uint8))
    g = N.PeerGroup(0, 2, 0, [A0.device_pointer, A1.device_pointer], ARENA)
    try:
        g.rowshard_matvec(N.Q4_K, W.device_pointer, X.device_pointer, 0, rows, cols, ctx.stream)
        ctx.synchronize()
        assert N.device_error_take(0) & ERR_PEER_TIMEOUT
        # this rank's half arrived in both arenas
        half = rows // 2
        y0 = A0.readback(4 * half).view(np.float32)
        y1 = A1.readback(4 * half).view(np.float32)
        np.testing.assert_array_equal(y0, y1)
        north_star_gate(y0, ref[:half], x, row_norm_max(N.Q4_K, blob, rows, cols), cols)
        # the context is still usable
        Y = ctx.buffer(4 * rows)
        W2 = ctx.buffer(blob.nbytes)
        W2.upload(blob)
        ctx.matvec(N.Q4_K, W2, X, Y, rows, cols)
        north_star_gate(Y.readback().view(np.float32), ref, x, row_norm_max(N.Q4_K, blob, rows, cols), cols)
        assert N.device_error_take(0) == 0
    finally:
        g.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    from sharpinference_b200 import native as nv
    ok = True
    msg = ""
    with nv.Context(rank) as c:
        arena = c.buffer(ARENA)
        handles = [None] * world
        dist.all_gather_object(handles, nv.ipc_export(arena.device_pointer))
        addrs = [arena.device_pointer if q == rank else nv.ipc_open(rank, handles[q]) for q in range(world)]
        g = nv.PeerGroup(rank, world, rank, addrs, ARENA)
        dist.barrier()
        for i, (wt, rows, cols) in enumerate([(nv.Q4_K, 5120, 3072), (nv.Q8_0, 7680, 5120), (nv.Q4_K, 200064, 3072)]):
            b, cnt, per = nv.rowshard_plan(rows, world, rank)
            shard = nv.synth_weight_rows(wt, 20 + i, b, cnt, cols, 0.02)
            x = nv.synth_normal(70 + i, cols, 1.0)
            W, X = c.buffer(shard.nbytes), c.buffer(4 * cols)
            W.upload(shard), X.upload(x)
            off = (i % 2) << 20 if rows * 4 <= (1 << 20) else 2 << 20
            g.rowshard_matvec(wt, W.device_pointer, X.device_pointer, off, rows, cols, c.stream)
            c.synchronize()
            y = arena.readback(4 * rows, offset=off).view(np.float32).copy()
            full = nv.synth_weights(wt, 20 + i, rows, cols, 0.02)
            ref = oracle.matvec(wt, full, x, rows, cols)
            rel = float(np.linalg.norm(y - ref) / np.linalg.norm(ref))
            if not rel <= 1e-4:
                ok, msg = False, f"shape {rows}x{cols}: rel {rel}"
            W.free(), X.free()
        err = nv.device_error_take(rank)
        if err:
            ok, msg = False, f"device error word {err}"
        dist.barrier()
        g.close()
        for q in range(world):
            if q != rank:
                nv.ipc_close(rank, addrs[q])
        dist.barrier()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write("ok" if ok else msg)
    dist.destroy_process_group()


def test_two_ranks_on_two_gpus(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    res = str(tmp_path / "res")
    mp.start_processes(_two_rank_worker, args=(2, _free_port(), res), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        assert open(f"{res}.{r}").read() == "ok"
