"""Sequence-split decode plumbing on two CPU ranks (gloo).

Each rank computes the oracle partial over its own slice of the positions, the
partials go through ``seqsplit.gather_merge`` (the same all-gather + merge step the
NCCL path uses) and the merged result must equal the single-rank oracle decode.
A second test drops a rank before the collective: the survivor must get an error
from the short process-group timeout instead of hanging.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mla_kv_quant_b200.seqsplit import gather_merge, rank_token_range
from oracle import codec, decode, writer


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make_pool(seed=3, d=256, dr=32, L=700):
    rng = np.random.default_rng(seed)
    pool = writer.Pool(num_slots=64 * 16, d=d, dr=dr, max_reqs=2, sink=4, recent=16)
    pt = np.array([[3, 1, 7, 2, 9, 4, 11, 5, 6, 8, 10]], np.int32)
    slots = decode.token_slots(pt[0], L)
    x = rng.standard_normal((L, d)).astype(np.float32)
    kpe = writer.bf16_bits(rng.standard_normal((L, dr)).astype(np.float32))
    writer.write(pool, x, kpe, slots, np.full(L, L), np.zeros(L, np.int64), *codec.serving_scalars(0.9, 1.05)[:2],
                 positions=np.arange(L))
    q = writer.bf16_bits(rng.standard_normal((1, 8, d + dr)).astype(np.float32))
    return pool, pt, slots, q, L


def _merge_np(parts_o, parts_lse):
    o, lse = decode.merge(parts_o.numpy().astype(np.float64), parts_lse.numpy().astype(np.float64))
    return torch.from_numpy(o), torch.from_numpy(lse)


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        pool, pt, slots, q, L = _make_pool()
        s, e = rank_token_range(L, world, rank)
        qf = writer.bf16_to_f32(q).astype(np.float64)[0]
        lat = decode.latent_rows(pool, slots, L)
        pe = writer.bf16_to_f32(pool.rope[slots]).astype(np.float64)
        o, lse = decode.attend(qf, lat[s:e], pe[s:e], 0.07)
        out, out_lse = gather_merge(torch.from_numpy(o).float(), torch.from_numpy(lse).float(), merge=_merge_np)
        result_q.put((rank, out.numpy(), out_lse.numpy()))
    except Exception as exc:
        result_q.put((rank, None, repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


def test_seqsplit_gather_merge_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, out, info in results:
        assert out is not None, f"rank {rank}: {info}"
    pool, pt, slots, qq, L = _make_pool()
    ref, ref_lse = decode.decode(pool, qq, pt, [L], 0.07)
    for _, out, lse in results:
        assert np.allclose(out, ref[0], atol=2e-5, rtol=1e-4)
        assert np.allclose(lse, ref_lse[0], atol=1e-5)


def _dropout_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        # leaves between steps: no collective of this step is ever joined
        result_q.put((rank, "left"))
        result_q.close()
        result_q.join_thread()
        os._exit(0)
    try:
        gather_merge(torch.zeros(4, 8), torch.zeros(4), merge=lambda o, l: (o[0], l[0]))
        result_q.put((rank, "completed"))
    except Exception as exc:  # the survivor learns of the missing rank from the timeout
        result_q.put((rank, f"error:{type(exc).__name__}"))


def test_seqsplit_rank_dropout_is_reported():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1] == "left"
    assert got[0].startswith("error:")
