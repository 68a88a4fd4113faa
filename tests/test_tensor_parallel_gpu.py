"""Tensor-parallel decoder session (si_decoder_create_tensor_parallel):
Megatron-style pairing, qkv / gate_up by rows of the rank's heads and
intermediate slice, out / down by columns with their partial vectors
exchanged through the peer arenas, heads-local attention. One rank on one
GPU (the whole code path, exchange included) and two ranks on two GPUs
(skipped on one GPU), against the oracle's greedy ids."""
import os
import socket

import numpy as np
import pytest

import oracle
from sharpinference_b200 import native, phi4
from test_transformer_oracle import tiny_decoder_config, tiny_decoder_weights

pytestmark = pytest.mark.gpu
N = native

MID_CFG = dict(layers=2, hidden=1024, query_heads=8, kv_heads=2, head_size=128, rotary_size=128, intermediate=2048,
               vocab=2048, context=64, epsilon=1e-5, rope_base=250000.0, rope_scale=1.0, weight_type=N.Q8_0,
               embedding_type=N.Q8_0)


def _arena_bytes(cfg, n):
    return (N.tp_arena_bytes(cfg, n) + 255) // 256 * 256


@pytest.mark.parametrize("wtype", [N.Q8_0, N.Q4_K])
def test_single_rank_tensor_parallel_session_matches_oracle(ctx, wtype):
    cfg = tiny_decoder_config(wtype)
    cfg["rotary_size"] = 128
    weights = tiny_decoder_weights(cfg, seed=71 + wtype)
    prompt = np.random.default_rng(71).integers(0, cfg["vocab"], 14)
    want = oracle.Decoder(cfg, weights).generate(prompt, 16)
    ab = _arena_bytes(cfg, 1)
    arena = ctx.buffer(ab)
    arena.upload(np.zeros(ab, np.uint8))
    group = N.PeerGroup(0, 1, 0, [arena.device_pointer], ab)
    try:
        with N.Decoder(cfg, 0, group, tensor_parallel=True) as dec:
            for name, arr in phi4.tp_slice_weights(cfg, weights, N.tp_partition(cfg, 1, 0)).items():
                dec.upload(name, arr)
            assert list(dec.generate(prompt, 16)) == want
            dec.reset()
            got, tok = [], None
            for i in range(30):
                tok = dec.forward_token(int(prompt[i]) if i < len(prompt) else tok)
                got.append(tok)
            assert got == want
        assert N.device_error_take(0) == 0
    finally:
        group.close()
        arena.free()


def test_tensor_parallel_rejects_small_arena_and_dense_types(ctx):
    cfg = tiny_decoder_config(N.Q8_0)
    ab = _arena_bytes(cfg, 1)
    arena = ctx.buffer(ab)
    small = N.PeerGroup(0, 1, 0, [arena.device_pointer], 4096 + 256)
    group = N.PeerGroup(0, 1, 0, [arena.device_pointer], ab)
    try:
        with pytest.raises(N.ArgumentError, match="arenas"):
            N.Decoder(cfg, 0, small, tensor_parallel=True)
        with pytest.raises(N.NotSupportedError):
            N.Decoder(dict(cfg, weight_type=N.F16), 0, group, tensor_parallel=True)
    finally:
        small.close()
        group.close()
        arena.free()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, prompt, steps, result_path):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(rank)
    from sharpinference_b200 import native as nv
    cfg = dict(MID_CFG)
    weights = tiny_decoder_weights(cfg, seed=87)
    ab = _arena_bytes(cfg, world)
    toks, msg = None, ""
    with nv.Context(rank) as c:
        arena = c.buffer(ab)
        arena.upload(np.zeros(ab, np.uint8))
        handles = [None] * world
        dist.all_gather_object(handles, nv.ipc_export(arena.device_pointer))
        addrs = [arena.device_pointer if q == rank else nv.ipc_open(rank, handles[q]) for q in range(world)]
        g = nv.PeerGroup(rank, world, rank, addrs, ab)
        try:
            with nv.Decoder(cfg, rank, g, tensor_parallel=True) as dec:
                part = nv.tp_partition(cfg, world, rank)
                for name, arr in phi4.tp_slice_weights(cfg, weights, part).items():
                    dec.upload(name, arr)
                dist.barrier()  # every arena mapped and every session built before the first step
                toks = [int(t) for t in dec.generate(prompt, steps)]
                err = nv.device_error_take(rank)
                if err:
                    msg = f"device error word {err}"
                dist.barrier()
        finally:
            g.close()
            for q in range(world):
                if q != rank:
                    nv.ipc_close(rank, addrs[q])
            dist.barrier()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write(msg or " ".join(map(str, toks)))
    dist.destroy_process_group()


def test_two_rank_tensor_parallel_session_matches_oracle(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    cfg = dict(MID_CFG)
    weights = tiny_decoder_weights(cfg, seed=87)
    prompt = [int(t) for t in np.random.default_rng(87).integers(0, cfg["vocab"], 12)]
    want = oracle.Decoder(cfg, weights).generate(prompt, 12)
    res = str(tmp_path / "res")
    mp.start_processes(_worker, args=(2, _free_port(), prompt, 12, res), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        got = open(f"{res}.{r}").read()
        assert got == " ".join(map(str, want)), f"rank {r}: {got}"
