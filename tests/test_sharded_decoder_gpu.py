"""Row-sharded decoder session (si_decoder_create_sharded, config 5's layout):
every projection holds one rank's rows and runs as the fused peer GEMV that
stores the rank's output rows into every rank's arena; the rest of the
decode program is replicated. One rank on one GPU (the arena path itself),
and two ranks on two GPUs (skipped on one GPU), both against the oracle's
greedy ids."""
import os
import socket

import numpy as np
import pytest

import oracle
from sharpinference_b200 import native
from test_transformer_oracle import tiny_decoder_config, tiny_decoder_weights

pytestmark = pytest.mark.gpu
N = native


def _row_bytes(wt, cols):
    return N.row_bytes(wt, cols)


def _shard_weights(cfg, weights, world, rank, dec=None):
    """This rank's rows of every split projection slot (all of them, or
    those the session split: a slot smaller than the whole matrix);
    token_embedding, the norms and replicated projections whole."""
    h, f = cfg["hidden"], cfg["intermediate"]
    qkv = h + 2 * cfg["kv_heads"] * cfg["head_size"]
    out = {}
    for name, arr in weights.items():
        base = name.rsplit("_", 1)[0]
        rows = {"qkv_weight": qkv, "attn_output_weight": h, "ffn_up_weight": 2 * f, "ffn_down_weight": h}.get(base)
        if rows is None:
            out[name] = arr
            continue
        cols = f if base == "ffn_down_weight" else h
        rb = _row_bytes(cfg["weight_type"], cols)
        if dec is not None and dec.slot(name)[1] == rows * rb:
            out[name] = arr  # replicated
            continue
        b, cnt, _ = N.rowshard_plan(rows, world, rank)
        out[name] = np.ascontiguousarray(arr.reshape(rows, rb)[b:b + cnt]).reshape(-1)
    return out


def _arena_bytes(cfg):
    return (N.decoder_arena_bytes(cfg) + 255) // 256 * 256


@pytest.mark.parametrize("wtype", [N.Q4_K, N.Q8_0])
def test_single_rank_sharded_session_matches_oracle(ctx, wtype):
    cfg = tiny_decoder_config(wtype)
    weights = tiny_decoder_weights(cfg, seed=61 + wtype)
    prompt = np.random.default_rng(61).integers(0, cfg["vocab"], 14)
    want = oracle.Decoder(cfg, weights).generate(prompt, 16)
    ab = _arena_bytes(cfg)
    arena = ctx.buffer(ab)
    group = N.PeerGroup(0, 1, 0, [arena.device_pointer], ab)
    try:
        with N.Decoder(cfg, 0, group) as dec:
            for name, arr in weights.items():
                dec.upload(name, arr)
            assert list(dec.generate(prompt, 16)) == want
            dec.reset()
            got, tok = [], None
            for i in range(30):
                tok = dec.forward_token(int(prompt[i]) if i < len(prompt) else tok)
                got.append(tok)
            assert got == want
            dec.reset()
            assert dec.prefill(prompt) == want[len(prompt) - 1]  # the decode program per token when sharded
        assert N.device_error_take(0) == 0
    finally:
        group.close()
        arena.free()


def test_sharded_session_rejects_small_arena_and_dense_types(ctx):
    cfg = tiny_decoder_config(N.Q4_K)
    ab = _arena_bytes(cfg)
    arena = ctx.buffer(ab)
    small = N.PeerGroup(0, 1, 0, [arena.device_pointer], 4096 + 256)
    group = N.PeerGroup(0, 1, 0, [arena.device_pointer], ab)
    try:
        with pytest.raises(N.ArgumentError, match="arenas"):
            N.Decoder(cfg, 0, small)
        dense = dict(cfg, weight_type=N.F16)
        with pytest.raises(N.NotSupportedError):
            N.Decoder(dense, 0, group)
    finally:
        small.close()
        group.close()
        arena.free()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


MID_CFG = dict(layers=2, hidden=1024, query_heads=8, kv_heads=2, head_size=128, rotary_size=128, intermediate=2048,
               vocab=2048, context=64, epsilon=1e-5, rope_base=250000.0, rope_scale=1.0, weight_type=N.Q8_0,
               embedding_type=N.Q8_0)


def _worker(rank, world, port, prompt, steps, result_path, shard_min_bytes=0):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(rank)
    from sharpinference_b200 import native as nv
    cfg = dict(MID_CFG)
    weights = tiny_decoder_weights(cfg, seed=83)
    ab = _arena_bytes(cfg)
    toks, msg = None, ""
    with nv.Context(rank) as c:
        arena = c.buffer(ab)
        arena.upload(np.zeros(ab, np.uint8))
        handles = [None] * world
        dist.all_gather_object(handles, nv.ipc_export(arena.device_pointer))
        addrs = [arena.device_pointer if q == rank else nv.ipc_open(rank, handles[q]) for q in range(world)]
        g = nv.PeerGroup(rank, world, rank, addrs, ab)
        try:
            with nv.Decoder(cfg, rank, g, shard_min_bytes=shard_min_bytes) as dec:
                for name, arr in _shard_weights(cfg, weights, world, rank, dec).items():
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


# 0: every projection split; 2 MB: qkv and o replicated (1.7 and 1.1 MB of
# Q8_0), ffn_up, ffn_down and the vocabulary projection split.
@pytest.mark.parametrize("shard_min_bytes", [0, 2 << 20])
def test_two_rank_sharded_session_matches_oracle(tmp_path, shard_min_bytes):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    cfg = dict(MID_CFG)
    weights = tiny_decoder_weights(cfg, seed=83)
    prompt = [int(t) for t in np.random.default_rng(83).integers(0, cfg["vocab"], 12)]
    want = oracle.Decoder(cfg, weights).generate(prompt, 12)
    res = str(tmp_path / "res")
    mp.start_processes(_worker, args=(2, _free_port(), prompt, 12, res, shard_min_bytes), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        got = open(f"{res}.{r}").read()
        assert got == " ".join(map(str, want)), f"rank {r}: {got}"
