"""gloo tests (world sizes 2 and 4) of the multi-GPU host logic on CPU: kv-head
sharding with the ctx all-gather, and sequence sharding, reproduce the unsharded
step."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from helpers import randn_half


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "tests"))
    import torch.distributed as dist

    from fully_custom_cuda_inference_lamma2_b200 import sharding
    from oracle import decode_oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, Hq, Hkv, D, cap = 3, 16, 4, 64, 40
        lens = torch.tensor([5, 30, 12], dtype=torch.int32)
        qq, kn, vn = randn_half((B, Hq, D), 1), randn_half((B, Hkv, D), 2), randn_half((B, Hkv, D), 3)
        kc, vc = randn_half((B, Hkv, cap, D), 4), randn_half((B, Hkv, cap, D), 5)
        full = O.decode_step(qq, kc, vc, lens, k_new=kn, v_new=vn)["ctx"]
        # kv-head shards + ctx all-gather
        kv_lo, kv_hi, q_lo, q_hi = sharding.partition_kv_heads(Hkv, Hq, world, rank)
        part = O.decode_step(qq[:, q_lo:q_hi], kc[:, kv_lo:kv_hi], vc[:, kv_lo:kv_hi], lens,
                             k_new=kn[:, kv_lo:kv_hi], v_new=vn[:, kv_lo:kv_hi])["ctx"]
        gathered = sharding.gather_ctx(part)
        ok_heads = torch.allclose(gathered, full, atol=1e-6)
        # the same into caller-owned buffers (nothing allocated per call)
        stage = torch.empty(world, B, q_hi - q_lo, D)
        out = torch.empty(B, Hq, D)
        sharding.gather_ctx(part, out=out, stage=stage)
        ok_heads = ok_heads and torch.allclose(out, full, atol=1e-6)
        # sequence shards: each rank computes its own sequences, results identical
        mine = sharding.partition_sequences(lens.tolist(), world)[rank]
        ok_seqs = True  # a rank may own no sequence when there are more ranks than sequences
        if mine:
            sub = O.decode_step(qq[mine], kc[mine], vc[mine], lens[mine], k_new=kn[mine], v_new=vn[mine])["ctx"]
            ok_seqs = torch.allclose(sub, full[mine], atol=1e-6)
        q.put((rank, bool(ok_heads), bool(ok_seqs), sorted(mine)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ranks_sharding_reproduces_unsharded(world):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok_h and ok_s for _, ok_h, ok_s, _ in results)
    covered = sorted(i for *_, mine in results for i in mine)
    assert covered == [0, 1, 2]
