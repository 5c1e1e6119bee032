"""The ctx exchange fused into the decode launch, on 2 to 4 GPUs of one node.

Each rank owns a kv-head shard; its decode launch stores the rank's ctx slice into
every rank's full-ctx buffer over NVLink (one plain store per peer, to CUDA IPC
mappings) and raises a per-rank flag; sharding.CtxExchange.wait() holds the stream
until every rank's slice has landed. Every rank's full ctx must match the fp32 oracle
of the unsharded step (max-abs 2e-3, relative-L2 1e-3) for three layers in a row
(alternating buffers), eagerly and replayed from a CUDA graph, with no timeout bit.
Runs as child processes, one per GPU, with NVLS off; skipped with fewer than 2 GPUs.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _cases(layers, B, Hq, Hkv, D, lens):
    from helpers import randn_half

    cap = max(lens) + 8
    out = []
    for l in range(layers):
        s = 100 * l
        out.append(dict(q=randn_half((B, Hq, D), s + 1), kn=randn_half((B, Hkv, D), s + 2),
                        vn=randn_half((B, Hkv, D), s + 3), kc=randn_half((B, Hkv, cap, D), s + 4),
                        vc=randn_half((B, Hkv, cap, D), s + 5)))
    return out


def _worker(rank, world, port, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "tests"))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    result = dict(rank=rank, ok=False, why="")
    try:
        import fully_custom_cuda_inference_lamma2_b200 as pkg
        from fully_custom_cuda_inference_lamma2_b200 import sharding
        from oracle import decode_oracle as O

        av = pkg.attn_varlen
        B, Hkv, G, D, layers = 4, 8, 8, 128, 3
        Hq = Hkv * G
        lens = [700, 65, 1500, 1]
        cases = _cases(layers, B, Hq, Hkv, D, lens)
        T = torch.tensor(lens, dtype=torch.int32)
        kv_lo, kv_hi, q_lo, q_hi = sharding.partition_kv_heads(Hkv, Hq, world, rank)
        ex = sharding.CtxExchange(B, Hq, D)
        shard = []
        for c in cases:
            shard.append(dict(q=c["q"][:, q_lo:q_hi].contiguous().to(dev),
                              kn=c["kn"][:, kv_lo:kv_hi].contiguous().to(dev),
                              vn=c["vn"][:, kv_lo:kv_hi].contiguous().to(dev),
                              kc=c["kc"][:, kv_lo:kv_hi].contiguous().to(dev),
                              vc=c["vc"][:, kv_lo:kv_hi].contiguous().to(dev)))
        want = [O.decode_step(c["q"], c["kc"], c["vc"], T, k_new=c["kn"], v_new=c["vn"])["ctx"] for c in cases]
        ws = av.make_workspace(B, q_hi - q_lo, kv_hi - kv_lo, D)
        lens_dev = T.to(dev)
        seq = lens_dev.clone()

        def step(check):
            errs = []
            for l, s in enumerate(shard):
                seq.copy_(lens_dev)
                full = ex.decode(s["q"], s["kc"], s["vc"], q_lo, l, k_new=s["kn"], v_new=s["vn"], seq_lens=seq,
                                 advance=True, workspace=ws, split=True)
                ex.wait()
                if check:
                    max_abs, rel = O.compare(full.float().cpu(), want[l])
                    errs.append((max_abs, rel))
            return errs

        errs = step(True)
        bad = [(l, e) for l, e in enumerate(errs) if not (e[0] <= O.MAX_ABS_TOL and e[1] <= O.REL_L2_TOL)]
        # the same three layers from one CUDA graph, replayed twice
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                step(False)
        torch.cuda.synchronize()
        dist.barrier()
        for _ in range(2):
            g.replay()
            torch.cuda.synchronize()
            dist.barrier()
        last = O.compare(ex.buffer(layers - 1).float().cpu(), want[layers - 1])
        if not (last[0] <= O.MAX_ABS_TOL and last[1] <= O.REL_L2_TOL):
            bad.append(("graph", last))
        err = ex.error() | av.read_error(ws)
        del g
        ex.close()
        result.update(ok=not bad and err == 0, why=f"bad={bad} err={err}")
    except Exception as e:  # reported to the parent, which fails the test
        result["why"] = repr(e)
    finally:
        q.put(result)
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ctx_exchange_fused_into_decode_matches_oracle():
    world = min(torch.cuda.device_count(), 4)
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    assert all(r["ok"] for r in results), results
    assert all(p.exitcode == 0 for p in procs)
