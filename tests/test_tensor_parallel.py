"""Tensor-parallel partition of the decode program (si_tp_partition_plan) and
the host-side slicing of the weights, on the CPU: every rank's slices are
disjoint and together rebuild the whole model, for config 5 (Phi-4-14B
shapes) over 1/2/4/8 ranks; world-size-2 gloo ranks plan and slice in
separate processes. The device path is tests/test_tensor_parallel_gpu.py."""
import datetime
import os
import socket

import numpy as np
import pytest

import oracle
from sharpinference_b200 import native, phi4

PHI4_14B = dict(layers=40, hidden=5120, query_heads=40, kv_heads=10, head_size=128, rotary_size=128,
                intermediate=17920, vocab=100352, context=4096, epsilon=1e-5, rope_base=250000.0, rope_scale=1.0,
                weight_type=native.Q8_0, embedding_type=native.Q8_0)
SMALL = dict(layers=1, hidden=1024, query_heads=8, kv_heads=4, head_size=128, rotary_size=128, intermediate=1536,
             vocab=700, context=32, epsilon=1e-5, rope_base=250000.0, rope_scale=1.0, weight_type=native.Q8_0,
             embedding_type=native.Q8_0)


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_partition_covers_config5_once(n):
    parts = [native.tp_partition(PHI4_14B, n, r) for r in range(n)]
    kv = sorted((p.kv_head_begin, p.kv_head_begin + p.kv_heads) for p in parts)
    assert kv[0][0] == 0 and kv[-1][1] == 10 and all(a[1] == b[0] for a, b in zip(kv, kv[1:]))
    assert all(p.query_head_begin == 4 * p.kv_head_begin and p.query_heads == 4 * p.kv_heads for p in parts)
    ffn = sorted((p.ffn_begin, p.ffn_begin + p.ffn_rows) for p in parts)
    assert ffn[0][0] == 0 and ffn[-1][1] == 17920 and all(a[1] == b[0] for a, b in zip(ffn, ffn[1:]))
    assert all(p.ffn_rows % 256 == 0 and p.ffn_rows > 0 for p in parts)
    voc = sorted((p.vocab_begin, p.vocab_begin + p.vocab_rows) for p in parts)
    assert voc[0][0] == 0 and voc[-1][1] == 100352 and all(a[1] == b[0] for a, b in zip(voc, voc[1:]))
    # the heaviest rank's weight bytes: about 1/n of the layer plus the uneven heads
    assert native.tp_arena_bytes(PHI4_14B, n) > n * 5120 * 4 * 2


def test_partition_rejects_unsplittable_layouts():
    with pytest.raises(native.NotSupportedError):
        native.tp_partition(PHI4_14B, 11, 0)  # more ranks than key/value heads
    mini = dict(PHI4_14B, hidden=3072, query_heads=24, kv_heads=8, intermediate=8192, weight_type=native.Q4_K,
                embedding_type=native.Q4_K)
    native.tp_partition(mini, 4, 1)  # 6 query heads = 768 columns: whole superblocks
    with pytest.raises(native.NotSupportedError):
        native.tp_partition(mini, 8, 0)  # 3 query heads = 384 columns of the out projection


def _small_model(seed=5):
    from test_transformer_oracle import tiny_decoder_weights
    return tiny_decoder_weights(SMALL, seed=seed)


def _reassemble(cfg, slices_by_rank, parts):
    """The whole model rebuilt from every rank's slices (inverse of tp_slice_weights)."""
    h, f, hs, kv = cfg["hidden"], cfg["intermediate"], cfg["head_size"], cfg["kv_heads"] * cfg["head_size"]
    wt = cfg["weight_type"]
    rbh, rbf = native.row_bytes(wt, h), native.row_bytes(wt, f)
    name_q, name_o, name_u, name_d = "qkv_weight_0", "attn_output_weight_0", "ffn_up_weight_0", "ffn_down_weight_0"
    qkv = np.zeros((h + 2 * kv, rbh), np.uint8)
    out = np.zeros((h, rbh), np.uint8)
    up = np.zeros((2 * f, rbh), np.uint8)
    down = np.zeros((h, rbf), np.uint8)
    for sl, p in zip(slices_by_rank, parts):
        q0, q1 = p.query_head_begin * hs, (p.query_head_begin + p.query_heads) * hs
        k0, k1 = p.kv_head_begin * hs, (p.kv_head_begin + p.kv_heads) * hs
        f0, f1 = p.ffn_begin, p.ffn_begin + p.ffn_rows
        m = sl[name_q].reshape(-1, rbh)
        nq, nk = q1 - q0, k1 - k0
        qkv[q0:q1], qkv[h + k0:h + k1], qkv[h + kv + k0:h + kv + k1] = m[:nq], m[nq:nq + nk], m[nq + nk:]
        b0, b1 = native.row_bytes(wt, q0) if q0 else 0, native.row_bytes(wt, q1)
        out[:, b0:b1] = sl[name_o].reshape(h, -1)
        u = sl[name_u].reshape(-1, rbh)
        up[f0:f1], up[f + f0:f + f1] = u[:f1 - f0], u[f1 - f0:]
        b0, b1 = native.row_bytes(wt, f0) if f0 else 0, native.row_bytes(wt, f1)
        down[:, b0:b1] = sl[name_d].reshape(h, -1)
    return {name_q: qkv.reshape(-1), name_o: out.reshape(-1), name_u: up.reshape(-1), name_d: down.reshape(-1)}


@pytest.mark.parametrize("n", [1, 2, 4])
def test_slices_rebuild_the_model(n):
    weights = _small_model()
    parts = [native.tp_partition(SMALL, n, r) for r in range(n)]
    slices = [phi4.tp_slice_weights(SMALL, weights, p) for p in parts]
    whole = _reassemble(SMALL, slices, parts)
    for name, arr in whole.items():
        assert np.array_equal(arr, weights[name]), name
    for sl in slices:  # norms and the table whole on every rank
        assert np.array_equal(sl["token_embedding"], weights["token_embedding"])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, out_path):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    part = native.tp_partition(SMALL, world, rank)
    sl = phi4.tp_slice_weights(SMALL, _small_model(), part)
    fields = [getattr(part, n) for n, _ in part._fields_]
    gathered = [None] * world
    dist.all_gather_object(gathered, (fields, {k: v.tobytes() for k, v in sl.items()}))
    if rank == 0:
        np.save(out_path, np.array(gathered, dtype=object), allow_pickle=True)
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_plan_and_slice(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "gathered.npy")
    mp.start_processes(_gloo_rank, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    gathered = np.load(out, allow_pickle=True)
    parts, slices = [], []
    for fields, sl in gathered:
        p = native.TpPartition(*fields)
        parts.append(p)
        slices.append({k: np.frombuffer(v, np.uint8) for k, v in sl.items()})
    assert [p.kv_head_begin for p in parts] == [0, 2] and [p.kv_heads for p in parts] == [2, 2]
    whole = _reassemble(SMALL, slices, parts)
    weights = _small_model()
    for name, arr in whole.items():
        assert np.array_equal(arr, weights[name]), name
