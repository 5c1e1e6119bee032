"""Decode-attention benchmark (B200): KV-read GB/s and tokens/s.

Workload (default `gqa70b`): the attention of one decode token for every layer of a
Llama-2-70B-shaped model — 80 layers, 64 query heads, 8 kv heads (GQA group 8),
head_dim 128, fp16 — for a batch of 32 sequences with 4096 cached keys each
(+1 appended per step), RoPE theta 1e4 on the new q/k. One step = for each layer,
one fused launch: RoPE(q, k_new) at T, append (k, v) at T, split-KV attention over
T+1 keys; the last layer's launch advances seq_len. Steps are replayed from one
CUDA graph; each step starts by restoring seq_len to 4096 (a 128-byte copy), so
every timed step has the configured shape. Synthetic data: K/V/q ~ N(0,1) fp16
from a seed; 43 GB of arena > the 126 MB L2, so no flush is needed between steps.

With --gpus N (one process per GPU under torchrun) the kv heads are sharded:
each rank owns 8/N kv heads and their 8 query heads each, for all 32 sequences
("strong" scaling: the whole job is fixed). `--gather-ctx` adds the NCCL
all-gather of ctx per layer that an unsharded output projection would need.

Other workloads: `gqa70b_32k` (batch 4 at 32768 keys), `varlen7b` (64 sequences,
lengths U[128, 8192], 32 heads, packed arena with cu_seqlens), `mha7b` (32 heads,
one sequence at 512 cached keys) — each with --layers — and `prefill16`: the causal
varlen prefill of 16 prompts of seeded lengths U[256, 4096] (32 heads, RoPE, arena
append, tcgen05 attention), reported in TFLOP/s of causal attention; `llama7b`: greedy
decode of a Llama-2-7B-shaped model (random weights, batch 1) with one CUDA graph per
token, in tokens/s (`--steps 484 --warmup 15` reproduces the 16 -> 516 KV range of the
reference's 500-token run).

`--impl reference` times the reference's own implementation of the path: its
attn_varlen CUDA kernel (built from the reference sources into oracle/_ref)
driven the way its decode driver drives it (torch RoPE and append per sequence,
contiguous slice + repeat_interleave, forward), on one layer of the workload
(a bounded sample), plus the torch-eager fp32 CPU oracle on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "decode-attn KV-read GB/s (% of HBM peak); tokens/s at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes need a profiler pass, which never runs inside a timed benchmark; the ncu
# captures of these kernels (commands and figures) are summarised under profiles/
TRAFFIC_NOTE = "not measured in this run: DRAM bytes come from separate ncu captures (profiles/)"


# ---------------------------------------------------------------- workloads

def workload(name: str, layers: int | None):
    if name == "gqa70b":
        w = dict(B=32, Hq=64, Hkv=8, D=128, lens=[4096] * 32, layers=80, packed=False)
    elif name == "gqa70b_32k":
        w = dict(B=4, Hq=64, Hkv=8, D=128, lens=[32768] * 4, layers=80, packed=False)
    elif name == "varlen7b":
        g = torch.Generator().manual_seed(3)
        lens = torch.randint(128, 8193, (64,), generator=g).tolist()
        w = dict(B=64, Hq=32, Hkv=32, D=128, lens=lens, layers=32, packed=True)
    elif name == "mha7b":
        w = dict(B=1, Hq=32, Hkv=32, D=128, lens=[512], layers=32, packed=False)
    else:
        raise SystemExit(f"unknown workload {name}")
    if layers is not None:
        w["layers"] = layers
    w["name"] = name
    return w


def with_kv_len(w, kv_len):
    """The workload with every sequence at kv_len cached keys (measurement sweeps)."""
    if kv_len:
        w = dict(w, lens=[kv_len] * w["B"], packed=False)
    return w


def algorithmic_bytes(B, Hq, Hkv, D, lens_plus1, append=True):
    """Bytes one launch must move: K+V of the attended keys, q in, ctx out, new rows in and out."""
    kv = sum(lens_plus1) * Hkv * D * 2 * 2
    qo = B * Hq * D * 2 * 2
    new = (B * Hkv * D * 2 * 2 * 2) if append else 0
    return kv + qo + new


def kv_read_bytes(Hkv, D, lens_plus1):
    return sum(lens_plus1) * Hkv * D * 2 * 2


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi sampling during the timed region (SM clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        if not getattr(self, "out", ""):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------- distributed

def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- our arm

def build_state(w, world, rank, seed=1234):
    import fully_custom_cuda_inference_lamma2_b200 as fcci
    from fully_custom_cuda_inference_lamma2_b200.sharding import partition_kv_heads, partition_sequences

    B, Hq, Hkv, D, L = w["B"], w["Hq"], w["Hkv"], w["D"], w["layers"]
    if w["packed"]:
        # sequences sharded across ranks
        seqs = partition_sequences(w["lens"], world)[rank]
        lens = [w["lens"][i] for i in seqs]
        hkv, hq = Hkv, Hq
        caps = [t + 1 for t in lens]
        arena = fcci.KVArena(L, len(lens), hkv, D, seq_capacities=caps, q_heads=hq)
    else:
        kv_lo, kv_hi, q_lo, q_hi = partition_kv_heads(Hkv, Hq, world, rank)
        hkv, hq = kv_hi - kv_lo, q_hi - q_lo
        q_lo_rank = q_lo
        lens = list(w["lens"])
        arena = fcci.KVArena(L, B, hkv, D, capacity=max(lens) + 1, q_heads=hq)
    b = len(lens)
    g = torch.Generator(device="cuda").manual_seed(seed + rank)
    for t in (arena.k, arena.v):
        flat = t.view(-1)
        chunk = 1 << 28
        for i in range(0, flat.numel(), chunk):
            flat[i:i + chunk].normal_(generator=g)
    lens_dev = torch.tensor(lens, dtype=torch.int32, device="cuda")
    arena.seq_lens.copy_(lens_dev)
    q = torch.randn(L, b, hq, D, generator=g, device="cuda").half()
    kn = torch.randn(L, b, hkv, D, generator=g, device="cuda").half()
    vn = torch.randn(L, b, hkv, D, generator=g, device="cuda").half()
    out = torch.empty(L, b, hq, D, dtype=torch.float16, device="cuda")
    return dict(fcci=fcci, arena=arena, lens=lens, lens_dev=lens_dev, q=q, kn=kn, vn=vn, out=out, hq=hq, hkv=hkv,
                b=b, q_lo=q_lo_rank if not w["packed"] else 0)


def run_step(st, gather=None):
    arena = st["arena"]
    arena.seq_lens.copy_(st["lens_dev"])
    L = arena.layers
    ex = st.get("exchange")
    for l in range(L):
        if ex is not None:
            # the launch stores its ctx slice into every rank's full-ctx buffer, then the
            # stream waits for every rank's slice of this layer
            k, v = arena.layer(l)
            ex.decode(st["q"][l], k, v, st["q_lo"], l, k_new=st["kn"][l], v_new=st["vn"][l],
                      seq_lens=arena.seq_lens, advance=(l == L - 1), workspace=arena.workspace, split=True,
                      prefetch_kv=st["prefetch_kv"])
            ex.wait()
            continue
        st["fcci"].decode_attention(arena, l, st["q"][l], st["out"][l], k_new=st["kn"][l], v_new=st["vn"][l],
                                    advance=(l == L - 1), prefetch_kv=st["prefetch_kv"])
        if gather is not None:
            gather(l)


def capture_step_graph(st, gather=None):
    """Two eager steps (kernel attributes, NCCL communicators), then one step captured."""
    for _ in range(2):
        run_step(st, gather)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream()
    cs.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cs):
        with torch.cuda.graph(graph, stream=cs):
            run_step(st, gather)
    torch.cuda.synchronize()
    return graph


def check_step(st, layer=0, out=None):
    """The timed step's answer at the timed shape: one layer's ctx of the last replay, on the
    first, middle and last sequence of this rank, against the fp32 oracle (max-abs 2e-3,
    relative-L2 1e-3). The appended row T is in the arena already; the oracle re-appends it."""
    sys.path.insert(0, ROOT)
    from oracle import decode_oracle as O

    arena = st["arena"]
    k, v = arena.layer(layer)
    picks = sorted({0, st["b"] // 2, st["b"] - 1})
    worst_abs, worst_rel = 0.0, 0.0
    for i in picks:
        T = st["lens"][i]
        if arena.packed:
            base = int(arena.cu_seqlens[i])
            kc = k[:, base:base + T + 1].unsqueeze(0).cpu()
            vc = v[:, base:base + T + 1].unsqueeze(0).cpu()
        else:
            kc, vc = k[i:i + 1, :, :T + 1].cpu(), v[i:i + 1, :, :T + 1].cpu()
        want = O.decode_step(st["q"][layer][i:i + 1].cpu(), kc, vc, torch.tensor([T], dtype=torch.int32),
                             k_new=st["kn"][layer][i:i + 1].cpu(), v_new=st["vn"][layer][i:i + 1].cpu(),
                             capacity=T + 1, inplace=True)
        got = (st["out"][layer] if out is None else out)[i:i + 1]
        ma, rel = O.compare(got.float().cpu(), want["ctx"])
        worst_abs, worst_rel = max(worst_abs, ma), max(worst_rel, rel)
    ok = worst_abs <= O.MAX_ABS_TOL and worst_rel <= O.REL_L2_TOL
    return {"ok": ok, "layer": layer, "sequences": picks, "max_abs": worst_abs, "rel_l2": worst_rel,
            "tolerance": {"max_abs": O.MAX_ABS_TOL, "rel_l2": O.REL_L2_TOL}}


def timed_replays(graph, steps, local):
    """K graph replays between events on the current stream, with the clock sampler running.
    K is raised so that the timed region lasts at least about 0.6 s (clock samples)."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    per = e0.elapsed_time(e1) / 3
    steps = max(steps, int(600.0 / max(per, 1e-3)) + 1)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    return e0.elapsed_time(e1), steps, clk.summary()


def decode_subrecord(name, layers, steps, local):
    """One decode workload on this GPU at its own shape (a fixed number of layers per step):
    KV GB/s, the kernel's roofline, clocks and the checked answer."""
    w = workload(name, layers)
    st = build_state(w, 1, 0)
    st["prefetch_kv"] = True
    graph = capture_step_graph(st)
    ms, steps, clocks = timed_replays(graph, steps, local)
    L, D = w["layers"], w["D"]
    lens1 = [t + 1 for t in st["lens"]]
    per_launch = algorithmic_bytes(st["b"], st["hq"], st["hkv"], D, lens1)
    launch_ms = ms / (steps * L)
    hbm, hbm_src = peaks()
    value = kv_read_bytes(st["hkv"], D, lens1) * L * steps / (ms / 1e3) / 1e9
    achieved = per_launch / (launch_ms / 1e3) / 1e9
    rec = {"workload": name, "value": round(value, 1), "unit": "GB/s", "layers": L, "steps": steps,
           "avg_launch_us": round(launch_ms * 1e3, 2),
           "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(achieved / hbm, 4), "peak_source": hbm_src, "traffic": None,
                        "algorithmic_bytes_per_launch": per_launch},
           "clocks": clocks, "checked": check_step(st)}
    del graph, st
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return rec


def mha7b_cpu_time(budget_s=3.0, seed=9):
    """The oracle's decode step of config 1 (one sequence, 32 heads, RoPE + append at T = 512,
    attention over 513 keys; torch fp32 eager) on the host cores: microseconds per step."""
    sys.path.insert(0, ROOT)
    from oracle import decode_oracle as O

    threads = cpu_threads()
    g = torch.Generator().manual_seed(seed)
    H, D, T = 32, 128, 512
    kc = torch.randn(1, H, T + 1, D, generator=g).half()
    vc = torch.randn(1, H, T + 1, D, generator=g).half()
    q, kn, vn = (torch.randn(1, H, D, generator=g).half() for _ in range(3))
    lens = torch.tensor([T], dtype=torch.int32)
    O.decode_step(q, kc, vc, lens, k_new=kn, v_new=vn, inplace=True)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        O.decode_step(q, kc, vc, lens, k_new=kn, v_new=vn, inplace=True)
        n += 1
    dt = time.perf_counter() - t0
    return {"us_per_step": round(dt / n * 1e6, 1), "cores": threads, "kind": "port",
            "sample": f"oracle decode_step (torch fp32 eager), B=1, 32 heads, T=512, {n} steps in {dt:.1f} s"}


def prefill_subrecord(local):
    """prefill16 (config 5) on this GPU, one layer per step: attention-kernel TFLOP/s and the
    whole step (RoPE + append + work list, then attention) against the dense peak."""
    w = prefill_workload("prefill16", 1)
    st = prefill_state(w, 1, 0)
    for _ in range(3):
        prefill_call(st, 0)
    torch.cuda.synchronize()
    K = 40
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        for e in ev:
            e[0].record()
            prefill_call(st, 0, "prepare")
            e[1].record()
            prefill_call(st, 0, "attend")
            e[2].record()
        torch.cuda.synchronize()
    step_ms = ev[0][0].elapsed_time(ev[-1][2]) / K
    attn_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / K
    prep_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / K
    fl = prefill_flops(w["Hq"], w["D"], st["lens"])
    peak, peak_src = tensor_peak()
    attn_tf, step_tf = fl / (attn_ms / 1e3) / 1e12, fl / (step_ms / 1e3) / 1e12
    rec = {"workload": "prefill16", "value": round(step_tf, 1), "unit": "TFLOP/s", "steps": K,
           "step_ms": round(step_ms, 4), "step_frac": round(step_tf / peak, 4),
           "roofline": {"bound": "tensor", "kernel": "prefill_attn_kernel", "achieved": round(attn_tf, 1),
                        "peak": peak, "unit": "TFLOP/s", "frac": round(attn_tf / peak, 4), "peak_source": peak_src,
                        "traffic": None, "algorithmic_flops_per_launch": fl, "avg_launch_ms": round(attn_ms, 5),
                        "prepare_avg_ms": round(prep_ms, 5)},
           "clocks": clk.summary()}
    del st
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return rec


def ours(args):
    world, rank, local = dist_setup(args.gpus)
    w = with_kv_len(workload(args.workload, args.layers), args.kv_len)
    if args.shard_of > 1 and world == 1:
        # one GPU runs rank 0's share of an N-way partition (for profiling that shape alone)
        st = build_state(w, args.shard_of, 0)
    else:
        st = build_state(w, world, rank)
    # each layer's launch may read its lengths and first K/V tiles while the previous
    # layer's launch drains: that launch writes only its own arena, ctx and workspace,
    # and only the last layer advances seq_lens (each step starts with a copy)
    st["prefetch_kv"] = not args.no_prefetch_kv
    L, D = w["layers"], w["D"]
    gather = None
    if args.gather_ctx and world > 1 and not w["packed"]:
        if args.gather_impl == "nccl":
            from fully_custom_cuda_inference_lamma2_b200.sharding import gather_ctx

            full = torch.empty(L, st["b"], w["Hq"], D, dtype=torch.float16, device="cuda")
            stage = torch.empty(world, st["b"], st["hq"], D, dtype=torch.float16, device="cuda")

            def gather(l):
                gather_ctx(st["out"][l], out=full[l], stage=stage)
        else:
            from fully_custom_cuda_inference_lamma2_b200.sharding import CtxExchange

            st["exchange"] = CtxExchange(st["b"], w["Hq"], D)

    graph = capture_step_graph(st, gather)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)

    lens1 = [t + 1 for t in st["lens"]]
    per_launch_alg = algorithmic_bytes(st["b"], st["hq"], st["hkv"], D, lens1)
    per_step_kv = kv_read_bytes(st["hkv"], D, lens1) * L
    # ---- timed region: K graph replays
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(world)
        torch.cuda.synchronize()
        ev0.record()
        for _ in range(args.steps):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize()
        barrier(world)
    ms_local = ev0.elapsed_time(ev1)
    ms = max_over_ranks(ms_local, world)
    ms_step = ms / args.steps
    kv_all = per_step_kv * args.steps
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([float(kv_all)], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        kv_all = float(t.item())
    value = kv_all / (ms / 1e3) / 1e9
    tokens_per_s = w["B"] * args.steps / (ms / 1e3)
    kernel_ms = ms_local / (args.steps * L)  # graph holds only the decode launches (+ one 128 B copy)
    achieved = per_launch_alg / (kernel_ms / 1e3) / 1e9
    hbm, hbm_src = peaks()
    clocks = clk.summary()

    # ---- the answer of the timed step, checked against the oracle on every rank (with the
    #      exchange, this rank's slice of the last layer's full-ctx buffer)
    ex = st.get("exchange")
    if ex is None:
        checked = check_step(st)
    else:
        checked = check_step(st, L - 1, ex.buffer(L - 1)[:, st["q_lo"]:st["q_lo"] + st["hq"]])
    ok_all = checked["ok"]
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([1.0 if ok_all else 0.0], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        ok_all = bool(t.item() > 0.5)

    # ---- e2e through the public API with host buffers (pinned), copies overlapped per layer
    e2e_line = None
    if not args.no_e2e:
        e2e = e2e_run(st, args, L)
        e2e_ms = max_over_ranks(e2e["ms"], world)
        e2e_kv = per_step_kv * e2e["steps"]
        if world > 1:
            import torch.distributed as dist

            t = torch.tensor([float(e2e_kv)], dtype=torch.float64, device="cuda")
            dist.all_reduce(t)
            e2e_kv = float(t.item())
        e2e_line = {"value": round(e2e_kv / (e2e_ms / 1e3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                    "ms_per_step": round(e2e_ms / e2e["steps"], 4), "api": e2e["api"],
                    "tokens_per_s": round(w["B"] * e2e["steps"] / (e2e_ms / 1e3), 1)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, budget_s=args.cpu_seconds)
    arena_gb = st["arena"].k.numel() * 4 / 1e9

    del graph
    barrier(world)
    if st.get("exchange") is not None:
        if st["exchange"].error():
            print("bench: the ctx exchange timed out on the device", file=sys.stderr, flush=True)
            ok_all = False
        st["exchange"].close()
    if not ok_all:
        if rank == 0:
            print(f"bench: the timed step's ctx differs from the oracle: {checked}", file=sys.stderr, flush=True)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        raise SystemExit(3)

    # ---- the other decode configurations and the prefill, each at its own shape (one GPU)
    sub = None
    if world == 1 and args.shard_of == 1 and w["name"] == "gqa70b" and not args.no_subrecords:
        del st
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        sub = {}
        for name, layers in (("gqa70b_32k", 20), ("varlen7b", 8), ("mha7b", 64)):
            sub[name] = decode_subrecord(name, layers, 10, local)
            if not sub[name]["checked"]["ok"]:
                print(f"bench: {name} ctx differs from the oracle: {sub[name]['checked']}", file=sys.stderr)
                raise SystemExit(3)
        if not args.no_cpu_baseline:
            sub["mha7b"]["cpu_fp32"] = mha7b_cpu_time()
        sub["prefill16"] = prefill_subrecord(local)

    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp16",
        "data": "synthetic (seeded N(0,1) fp16 K/V/q; random-init, no checkpoint)",
        "config": {
            "workload": w["name"], "batch": w["B"], "q_heads": w["Hq"], "kv_heads": w["Hkv"], "head_dim": D,
            "kv_len": (w["lens"][0] if len(set(w["lens"])) == 1 else "seeded U[128,8192]"), "layers": L,
            "parallelism": ("kv-head shards x%d" % world) if not w["packed"] else ("sequence shards x%d" % world),
            "shard_of": args.shard_of if world == 1 and args.shard_of > 1 else None,
            "gather_ctx": (args.gather_impl if args.gather_ctx and world > 1 and not w["packed"] else False),
            "prefetch_kv": not args.no_prefetch_kv,
            "max_cluster": args.max_cluster or "auto",
            "l2": "no flush: arena %.1f GB per GPU > 126 MB L2" % arena_gb,
        },
        "tokens_per_s": round(tokens_per_s, 1),
        "hbm_frac": round(value / world / hbm, 4),
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(achieved / hbm, 4), "peak_source": hbm_src,
            "traffic": None,
            "traffic_note": TRAFFIC_NOTE,
            "kernel": "decode_attn_kernel<128,1>", "algorithmic_bytes_per_launch": per_launch_alg,
            "avg_launch_ms": round(kernel_ms, 5),
        },
        "e2e": e2e_line,
        "gpu_launches": args.steps * L,
        "clocks": clocks,
        "checked": checked,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if sub is not None:
        line["configs"] = sub
    print(json.dumps(line), flush=True)


def e2e_run(st, args, L):
    """Per step: pinned-host q/k_new/v_new -> device (copy stream, one layer ahead),
    decode through attn_varlen.decode, ctx -> pinned host; timed with events. The step
    (copies and launches) is captured once and replayed as a CUDA graph, as the
    reference's capture/replay server runs its steps; eager calls when capture fails."""
    arena = st["arena"]
    hq = st["q"].cpu().pin_memory()
    hkn = st["kn"].cpu().pin_memory()
    hvn = st["vn"].cpu().pin_memory()
    hout = torch.empty(st["out"].shape, dtype=torch.float16).pin_memory()
    dq, dkn, dvn, dout = st["q"], st["kn"], st["vn"], st["out"]
    comp = torch.cuda.Stream()
    comp.wait_stream(torch.cuda.current_stream())
    copy_in = torch.cuda.Stream()
    copy_out = torch.cuda.Stream()
    steps = max(3, min(args.steps, 10))
    h2d = (hq.numel() + hkn.numel() + hvn.numel()) * 2
    d2h = hout.numel() * 2

    def one_step():
        arena.seq_lens.copy_(st["lens_dev"])
        ready = [torch.cuda.Event() for _ in range(L)]
        done = [torch.cuda.Event() for _ in range(L)]
        copy_in.wait_stream(comp)
        for l in range(L):
            with torch.cuda.stream(copy_in):
                dq[l].copy_(hq[l], non_blocking=True)
                dkn[l].copy_(hkn[l], non_blocking=True)
                dvn[l].copy_(hvn[l], non_blocking=True)
                ready[l].record(copy_in)
        for l in range(L):
            comp.wait_event(ready[l])
            st["fcci"].decode_attention(arena, l, dq[l], dout[l], k_new=dkn[l], v_new=dvn[l], advance=(l == L - 1),
                                        prefetch_kv=st["prefetch_kv"])
            done[l].record(comp)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(done[l])
                hout[l].copy_(dout[l], non_blocking=True)
        comp.wait_stream(copy_out)

    with torch.cuda.stream(comp):
        for _ in range(2):
            one_step()
    torch.cuda.synchronize()
    graph, api = None, "CUDA graph of the step: host copies and attn_varlen.decode per layer"
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=comp):
            one_step()
        torch.cuda.synchronize()
        graph = g
    except Exception as exc:  # keep the e2e leg: eager calls, as a user without graphs makes them
        torch.cuda.synchronize()
        api = "attn_varlen.decode per layer, eager (graph capture failed: %s)" % str(exc).splitlines()[0][:80]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(comp):
        if graph is not None:
            graph.replay()
        else:
            one_step()
        e0.record(comp)
        for _ in range(steps):
            if graph is not None:
                graph.replay()
            else:
                one_step()
        e1.record(comp)
    torch.cuda.synchronize()
    got = hout.to(torch.float32)
    if not torch.equal(hout[-1], st["out"][-1].cpu()) or not torch.isfinite(got).all():
        raise SystemExit("e2e: the ctx copied to the host differs from the device result")
    return {"ms": e0.elapsed_time(e1), "steps": steps, "h2d": h2d, "d2h": d2h, "api": api}


# ---------------------------------------------------------------- CPU oracle baseline

def cpu_threads():
    try:
        cores = len(os.sched_getaffinity(0))
    except AttributeError:
        cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    return torch.get_num_threads()


def cpu_baseline(w, budget_s=10.0, seed=7):
    """The torch-eager fp32 oracle on the host cores over a bounded sample: one layer's
    decode step for as many sequences as fit the time budget (whole steps)."""
    sys.path.insert(0, ROOT)
    from oracle import decode_oracle as O

    threads = cpu_threads()
    B, Hq, Hkv, D = w["B"], w["Hq"], w["Hkv"], w["D"]
    nseq = min(B, 4)
    lens = w["lens"][:nseq]
    g = torch.Generator().manual_seed(seed)
    cap = max(lens) + 1
    kc = torch.randn(nseq, Hkv, cap, D, generator=g).half()
    vc = torch.randn(nseq, Hkv, cap, D, generator=g).half()
    q = torch.randn(nseq, Hq, D, generator=g).half()
    kn = torch.randn(nseq, Hkv, D, generator=g).half()
    vn = torch.randn(nseq, Hkv, D, generator=g).half()
    T = torch.tensor(lens, dtype=torch.int32)
    O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn, inplace=True)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn, inplace=True)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    kv = kv_read_bytes(Hkv, D, [t + 1 for t in lens]) * n
    return {"value": round(kv / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"oracle decode_step (torch fp32 eager) on {nseq} of {B} sequences x 1 layer, "
                      f"{n} repetitions in {dt:.1f} s",
            "tokens_per_s": round(nseq * n / dt, 2)}


# ---------------------------------------------------------------- prefill (causal varlen, tcgen05)

PREFILL_METRIC = "causal varlen prefill TFLOP/s (RoPE + arena append + attention), fraction of dense fp16 peak"


def prefill_workload(name: str, layers: int | None):
    """prefill16: 16 prompts of seeded lengths U[256, 4096], 32 heads (MHA), head_dim 128."""
    g = torch.Generator().manual_seed(5)
    lens = torch.randint(256, 4097, (16,), generator=g).tolist()
    return dict(name=name, B=16, Hq=32, Hkv=32, D=128, lens=lens, layers=layers or 1)


def prefill_flops(Hq, D, lens):
    """4 * Hq * D per (query, visible key) pair: QK^T and PV, causal (keys <= position)."""
    return sum(4 * Hq * D * (L * (L + 1) // 2) for L in lens)


def tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured (cuBLAS bf16 burst; fp16 runs at the same rate)"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def prefill_state(w, world, rank, seed=99):
    import fully_custom_cuda_inference_lamma2_b200 as fcci
    from fully_custom_cuda_inference_lamma2_b200.sharding import partition_by_cost

    seqs = partition_by_cost([L * (L + 1) / 2 for L in w["lens"]], world)[rank]
    lens = [w["lens"][i] for i in seqs]
    Hq, Hkv, D, layers = w["Hq"], w["Hkv"], w["D"], w["layers"]
    total, B = sum(lens), len(lens)
    cap = (max(lens) + 127) // 128 * 128
    g = torch.Generator(device="cuda").manual_seed(seed + rank)
    q = torch.randn(layers, total, Hq, D, generator=g, device="cuda").half()
    kn = torch.randn(layers, total, Hkv, D, generator=g, device="cuda").half()
    vn = torch.randn(layers, total, Hkv, D, generator=g, device="cuda").half()
    kc = torch.empty(layers, B, Hkv, cap, D, dtype=torch.float16, device="cuda")
    vc = torch.empty_like(kc)
    out = torch.empty(layers, total, Hq, D, dtype=torch.float16, device="cuda")
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    av = fcci.attn_varlen
    ws = av.make_prefill_workspace(B, Hq, Hkv, D, total, max(lens), cap)
    return dict(av=av, lens=lens, q=q, kn=kn, vn=vn, kc=kc, vc=vc, out=out, cu=cu, ws=ws, max_q=max(lens),
                layers=layers, B=B)


def prefill_call(st, l, part="all", q=None, kn=None, vn=None, out=None):
    st["av"].prefill_varlen(st["q"][l] if q is None else q, st["kn"][l] if kn is None else kn,
                            st["vn"][l] if vn is None else vn, st["kc"][l], st["vc"][l],
                            st["out"][l] if out is None else out, st["cu"], st["max_q"], fixed_len=0,
                            workspace=st["ws"], part=part)


def prefill_cpu_baseline(w, budget_s=10.0, seed=8):
    """The torch-eager fp32 oracle's prefill_step on the host cores, on a bounded sample:
    one prompt of 512 tokens x all heads, repeated for about budget_s."""
    sys.path.insert(0, ROOT)
    from oracle import decode_oracle as O

    threads = cpu_threads()
    Hq, Hkv, D, n = w["Hq"], w["Hkv"], w["D"], 512
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(n, Hq, D, generator=g).half()
    kn = torch.randn(n, Hkv, D, generator=g).half()
    vn = torch.randn(n, Hkv, D, generator=g).half()
    kc = torch.zeros(1, Hkv, n, D, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    cu, T = torch.tensor([0, n]), torch.tensor([0])
    O.prefill_step(q, kn, vn, kc, vc, cu, T)  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        O.prefill_step(q, kn, vn, kc, vc, cu, T)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    fl = prefill_flops(Hq, D, [n]) * reps
    return {"value": round(fl / dt / 1e12, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"oracle prefill_step (torch fp32 eager) on one {n}-token prompt x {Hq} heads, "
                      f"{reps} repetitions in {dt:.1f} s"}


def prefill_ours(args):
    world, rank, local = dist_setup(args.gpus)
    w = prefill_workload(args.workload, args.layers)
    st = prefill_state(w, world, rank)
    L = st["layers"]
    flops_step = prefill_flops(w["Hq"], w["D"], st["lens"]) * L
    for i in range(args.warmup):
        for l in range(L):
            prefill_call(st, l)
    torch.cuda.synchronize()
    barrier(world)
    K = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K * L)]
    with ClockSampler(local) as clk:
        barrier(world)
        torch.cuda.synchronize()
        for i in range(K):
            for l in range(L):
                e = ev[i * L + l]
                e[0].record()
                prefill_call(st, l, "prepare")
                e[1].record()
                prefill_call(st, l, "attend")
                e[2].record()
        torch.cuda.synchronize()
        barrier(world)
    ms_local = ev[0][0].elapsed_time(ev[-1][2])
    ms = max_over_ranks(ms_local, world)
    attn_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / len(ev)
    prep_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / len(ev)
    flops_all = flops_step * K
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([float(flops_all)], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        flops_all = float(t.item())
    value = flops_all / (ms / 1e3) / 1e12
    peak, peak_src = tensor_peak()
    per_launch = prefill_flops(w["Hq"], w["D"], st["lens"])
    achieved = per_launch / (attn_ms / 1e3) / 1e12
    clocks = clk.summary()

    # e2e through the public call with host buffers: per step and layer, the new
    # tokens' q/k/v go host -> device (pinned), the step runs, out goes device -> host
    hq, hk, hv = st["q"][0].cpu().pin_memory(), st["kn"][0].cpu().pin_memory(), st["vn"][0].cpu().pin_memory()
    ho = torch.empty(st["out"][0].shape, dtype=torch.float16).pin_memory()
    dq, dk, dv, do = st["q"][0], st["kn"][0], st["vn"][0], st["out"][0]
    e2e_steps = max(3, min(K, 5))
    for _ in range(2):
        dq.copy_(hq, non_blocking=True)
        prefill_call(st, 0, q=dq, kn=dk, vn=dv, out=do)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        for l in range(L):
            dq.copy_(hq, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            prefill_call(st, 0, q=dq, kn=dk, vn=dv, out=do)
            ho.copy_(do, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e_flops = flops_step * e2e_steps
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([float(e2e_flops)], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        e2e_flops = float(t.item())
    h2d = (hq.numel() + hk.numel() + hv.numel()) * 2 * L
    d2h = ho.numel() * 2 * L
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = prefill_cpu_baseline(w, budget_s=args.cpu_seconds)
    barrier(world)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return
    tokens = sum(w["lens"])
    line = {
        "metric": PREFILL_METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": round(ms / K, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp16",
        "data": "synthetic (seeded N(0,1) fp16 q/k/v; random-init, no checkpoint)",
        "config": {"workload": w["name"], "batch": w["B"], "q_heads": w["Hq"], "kv_heads": w["Hkv"],
                   "head_dim": w["D"], "prompt_lens": "seeded U[256,4096]", "tokens": tokens, "layers": L,
                   "causal": True, "parallelism": f"sequence shards x{world}",
                   "l2": "no flush: %.2f GB of q/k/v/arena per layer > 126 MB L2" % (
                       (st["q"][0].numel() * 3 + st["kc"][0].numel() * 2) * 2 / 1e9)},
        "tokens_per_s": round(tokens * K * L / (ms / 1e3), 1),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_src,
                     "traffic": None,
                     "traffic_note": TRAFFIC_NOTE,
                     "kernel": "prefill_attn_kernel", "algorithmic_flops_per_launch": per_launch,
                     "avg_launch_ms": round(attn_ms, 5), "prepare_avg_ms": round(prep_ms, 5)},
        "e2e": {"value": round(e2e_flops / (e2e_ms / 1e3) / 1e12, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / e2e_steps, 4),
                "api": "attn_varlen.prefill_varlen per layer, host q/k/v in, host out"},
        "gpu_launches": K * L * 2,
        "clocks": clocks,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def prefill_reference(args):
    """The reference's prefill of one layer as its kv_init runs it: one HF model forward per
    prompt (batch 1) - LlamaRotaryEmbedding + apply_rotary_pos_emb in fp16 and the causal
    SDPA attention it selects (attn_implementation "sdpa") - then the copy of the rotated
    keys and the values into the arena rows, per prompt, on the GPU."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    try:
        from transformers import LlamaConfig
        from transformers.integrations.sdpa_attention import sdpa_attention_forward
        from transformers.models.llama import modeling_llama as M
    except Exception as e:  # transformers missing or changed
        print(json.dumps({"impl": "reference", "unavailable": f"transformers Llama functions: {e}"}), flush=True)
        return
    w = prefill_workload(args.workload, args.layers)
    Hq, Hkv, D, lens = w["Hq"], w["Hkv"], w["D"], w["lens"]
    cap = (max(lens) + 127) // 128 * 128
    cfg = LlamaConfig(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=Hkv, head_dim=D,
                      max_position_embeddings=cap, rope_theta=10000.0)
    rope = M.LlamaRotaryEmbedding(cfg).cuda()

    class _Mod(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.num_key_value_groups = Hq // Hkv
            self.is_causal = True
            self.training = False

    mod = _Mod()
    g = torch.Generator(device="cuda").manual_seed(99)
    qs = [torch.randn(1, Hq, L, D, generator=g, device="cuda").half() for L in lens]
    ks = [torch.randn(1, Hkv, L, D, generator=g, device="cuda").half() for L in lens]
    vs = [torch.randn(1, Hkv, L, D, generator=g, device="cuda").half() for L in lens]
    arena_k = torch.empty(len(lens), Hkv, cap, D, dtype=torch.float16, device="cuda")
    arena_v = torch.empty_like(arena_k)
    x = torch.empty(1, 1, Hq * D, dtype=torch.float16, device="cuda")

    def one_step():
        for b, L in enumerate(lens):
            pos = torch.arange(L, device="cuda").view(1, -1)
            cos, sin = rope(x, pos)
            q, k = M.apply_rotary_pos_emb(qs[b], ks[b], cos, sin)
            sdpa_attention_forward(mod, q, k, vs[b], None, scaling=D ** -0.5, is_causal=True)
            arena_k[b, :, :L].copy_(k[0])
            arena_v[b, :, :L].copy_(vs[b][0])

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        one_step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    fl = prefill_flops(Hq, D, lens) * args.steps
    value = fl / (ms / 1e3) / 1e12
    cpu = prefill_cpu_baseline(w, budget_s=args.cpu_seconds) if not args.no_cpu_baseline else None
    line = {"impl": "reference", "metric": PREFILL_METRIC, "value": round(value, 2), "unit": "TFLOP/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (seeded N(0,1) fp16 q/k/v)",
            "config": {"workload": w["name"], "batch": w["B"], "q_heads": Hq, "kv_heads": Hkv, "head_dim": D,
                       "prompt_lens": "seeded U[256,4096]", "layers": 1, "causal": True,
                       "path": "HF LlamaRotaryEmbedding + apply_rotary_pos_emb + sdpa_attention_forward per "
                               "prompt, arena copy (case4_graph_generator_server_ipc.py:1241-1262)"},
            "e2e": {"value": round(value, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if world > 1:
        line["note"] = f"rank 0 of {world} ran the single-GPU reference; other ranks idle"
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- Llama-2-7B greedy decode (config 2)

LLAMA_METRIC = "Llama-2-7B-shaped greedy decode tokens/s, batch 1 (fraction of the weight-read HBM bound)"


def llama_ours(args):
    """Prompt of 16 seeded tokens through the prefill path, then `steps` timed greedy tokens, one
    CUDA-graph replay each (all 32 layers, device-side length). With the warm-up tokens the KV
    length goes from 16 to 16 + warmup + steps (516 with the defaults)."""
    world, rank, local = dist_setup(args.gpus)
    from fully_custom_cuda_inference_lamma2_b200.llama_decode import LLAMA2_7B, GreedyDecoder, LlamaWeights

    s = LLAMA2_7B
    W, K = args.warmup, args.steps
    prompt_len = 16
    new = 1 + W + K
    w = LlamaWeights(s, seed=11 + rank)
    dec = GreedyDecoder(w, capacity=prompt_len + new + 8, max_new_tokens=new + 1)
    prompt = torch.randint(0, s.vocab, (prompt_len,), generator=torch.Generator().manual_seed(12)).cuda()
    dec.arena.seq_lens.zero_()
    dec.step_idx.zero_()
    dec.prefill(prompt)
    dec.generated[0:1].copy_(dec.token)
    dec.step_idx.fill_(1)
    dec.capture()
    for _ in range(W):
        dec.graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(world)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(K):
            dec.graph.replay()
        e1.record()
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    tok_s = K * world / (ms / 1e3)
    hbm, hbm_src = peaks()
    step_bytes = s.weight_bytes()
    achieved = step_bytes / (ms / K / 1e3) / 1e9
    final_len = int(dec.arena.seq_lens.item())
    # e2e: the serving loop's host round trip per token (token id in from pinned host memory,
    # next id back to the host), through the same graph
    h_in = torch.zeros(1, dtype=torch.int64).pin_memory()
    h_out = torch.zeros(1, dtype=torch.int64).pin_memory()
    h_in.copy_(dec.token.cpu())
    dec.arena.seq_lens.fill_(prompt_len)  # the same KV range again, from the prompt on
    dec.step_idx.fill_(1)
    e2e_steps = min(K, 100)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(e2e_steps):
        dec.token.copy_(h_in, non_blocking=True)
        dec.graph.replay()
        h_out.copy_(dec.token, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        h_in.copy_(h_out)
    t1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(t0.elapsed_time(t1), world)
    barrier(world)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": LLAMA_METRIC, "value": round(tok_s, 2), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": round(ms / K, 4), "higher_is_better": True,
        "scaling": "weak" if world > 1 else "strong", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (random-init N(0,0.02) weights from a seed, 16 seeded prompt tokens; no checkpoint)",
        "config": {"workload": "llama7b", "layers": s.layers, "hidden": s.hidden, "heads": s.heads,
                   "intermediate": s.intermediate, "vocab": s.vocab, "batch": 1, "prompt": prompt_len,
                   "kv_len": f"{prompt_len + 1 + W} -> {final_len}", "graphs": "one graph for every length",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "no flush: 13.2 GB of weights per step > 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_source": hbm_src, "traffic": None,
                     "kernel": "whole token step (fused gemv_kernel projections + decode_attn_kernel; RMSNorm/SwiGLU/residual fused)",
                     "algorithmic_bytes_per_step": step_bytes, "avg_step_ms": round(ms / K, 5)},
        "e2e": {"value": round(e2e_steps / (e2e_ms / 1e3), 2), "unit": "tokens/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 8, "api": "graph replay per token, token id host->device and back"},
        "gpu_launches": K * (s.layers * 4 + 1),  # this library's kernels: 2 RMSNorm, decode, SwiGLU per layer; final RMSNorm
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def llama_reference(args):
    """The reference's decode of config 2 as it publishes it: HF LlamaForCausalLM greedy
    generation with its KV cache (fp16, sdpa attention), same shapes, random-init weights."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    try:
        from transformers import LlamaConfig, LlamaForCausalLM
    except Exception as e:
        print(json.dumps({"impl": "reference", "unavailable": f"transformers Llama: {e}"}), flush=True)
        return
    W, K = args.warmup, args.steps
    cfg = LlamaConfig(hidden_size=4096, intermediate_size=11008, num_hidden_layers=32, num_attention_heads=32,
                      num_key_value_heads=32, vocab_size=32000, rms_norm_eps=1e-5, tie_word_embeddings=True,
                      rope_theta=10000.0, max_position_embeddings=4096)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(13)
    with torch.device("cuda"):
        model = LlamaForCausalLM(cfg).half().eval()
    prompt = torch.randint(0, 32000, (1, 16), generator=torch.Generator().manual_seed(12)).cuda()
    gen = dict(do_sample=False, eos_token_id=None, pad_token_id=0)
    with torch.no_grad():
        model.generate(prompt, max_new_tokens=W, min_new_tokens=W, **gen)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = model.generate(prompt, max_new_tokens=K, min_new_tokens=K, **gen)
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    n = out.shape[1] - prompt.shape[1]
    value = n / (ms / 1e3)
    print(json.dumps({"impl": "reference", "metric": LLAMA_METRIC, "value": round(value, 2), "unit": "tokens/s",
                      "n_gpus": 1, "steps": K, "warmup": W, "ms_per_step": round(ms / n, 4),
                      "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
                      "data": "synthetic (random-init weights, seeded prompt)",
                      "config": {"workload": "llama7b", "batch": 1, "prompt": 16,
                                 "path": "HF LlamaForCausalLM.generate, greedy, KV cache, sdpa (the reference's "
                                         "published decode path)"},
                      "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)


# ---------------------------------------------------------------- reference arm

def reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    sys.path.insert(0, ROOT)
    w = workload(args.workload, args.layers)
    try:
        import refkernels

        refkernels.ref_attn_varlen()
    except (OSError, FileNotFoundError) as exc:
        print(json.dumps({"impl": "reference", "unavailable": f"reference kernel not built: {exc}"}), flush=True)
        return
    from oracle import decode_oracle as O  # noqa: F401  (CPU leg below)

    B, Hq, Hkv, D = w["B"], w["Hq"], w["Hkv"], w["D"]
    G = Hq // Hkv
    lens = w["lens"]
    dev = "cuda"
    gen = torch.Generator(device=dev).manual_seed(99)
    cap = max(lens) + 1
    # one layer of the workload: the reference driver's per-sequence steps
    if w["packed"]:
        arena_k = [torch.randn(Hkv, t + 1, D, generator=gen, device=dev).half() for t in lens]
        arena_v = [torch.randn(Hkv, t + 1, D, generator=gen, device=dev).half() for t in lens]
    else:
        arena_k = [torch.randn(Hkv, cap, D, generator=gen, device=dev).half() for _ in range(B)]
        arena_v = [torch.randn(Hkv, cap, D, generator=gen, device=dev).half() for _ in range(B)]
    q = torch.randn(B, Hq, D, generator=gen, device=dev).half()
    kn = torch.randn(B, Hkv, D, generator=gen, device=dev).half()
    vn = torch.randn(B, Hkv, D, generator=gen, device=dev).half()
    scale = 1.0 / math.sqrt(D)
    inv = (10000.0 ** (-torch.arange(D // 2, device=dev, dtype=torch.float32) / float(D // 2))).view(1, -1)

    def rope_(hd, pos):  # the driver's apply_rope_ math, on the device as it runs it
        half = D // 2
        ang = pos * inv
        c, s = torch.cos(ang), torch.sin(ang)
        x1, x2 = hd[:, :half].float(), hd[:, half:].float()
        r1, r2 = (x1 * c - x2 * s).to(hd.dtype), (x2 * c + x1 * s).to(hd.dtype)
        hd[:, :half] = r1
        hd[:, half:] = r2
        return hd

    def layer_step(kernel_only_ms=None):
        for b in range(B):
            T = lens[b]
            qh = rope_(q[b].clone(), T)
            kh = rope_(kn[b].clone(), T)
            arena_k[b][:, T].copy_(kh)
            arena_v[b][:, T].copy_(vn[b])
            Ks = arena_k[b][:, :T + 1].contiguous().repeat_interleave(G, dim=0)
            Vs = arena_v[b][:, :T + 1].contiguous().repeat_interleave(G, dim=0)
            refkernels.ref_forward(qh, Ks, Vs, T + 1, scale)

    layer_step()
    torch.cuda.synchronize()
    steps = max(1, args.steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(args.warmup):
        layer_step()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        layer_step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    lens1 = [t + 1 for t in lens]
    kv = kv_read_bytes(Hkv, D, lens1) * steps
    value = kv / (ms / 1e3) / 1e9
    # kernel alone on pre-built inputs (first sequence), for context
    T = lens[0]
    Ks = arena_k[0][:, :T + 1].contiguous().repeat_interleave(G, dim=0)
    Vs = arena_v[0][:, :T + 1].contiguous().repeat_interleave(G, dim=0)
    qh = q[0].clone()
    refkernels.ref_forward(qh, Ks, Vs, T + 1, scale)
    torch.cuda.synchronize()
    e0.record()
    reps = 5
    for _ in range(reps):
        refkernels.ref_forward(qh, Ks, Vs, T + 1, scale)
    e1.record()
    torch.cuda.synchronize()
    k_ms = e0.elapsed_time(e1) / reps
    k_gbs = kv_read_bytes(Hkv, D, [T + 1]) / (k_ms / 1e3) / 1e9
    cpu = cpu_baseline(w, budget_s=args.cpu_seconds) if not args.no_cpu_baseline else None
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / steps, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp16",
        "data": "synthetic (seeded N(0,1) fp16)",
        "config": {"workload": w["name"], "batch": B, "q_heads": Hq, "kv_heads": Hkv, "head_dim": D,
                   "layers_timed_per_step": 1, "layers": w["layers"],
                   "sample": "one layer of the workload per step (bounded sample)"},
        "tokens_per_s_per_layer": round(B * steps / (ms / 1e3), 2),
        "implementation": ("reference custom_kernels/attn_varlen_kernel.cu built from source for sm_100a "
                           "(oracle/_ref), driven as scripts/direct_custom_decode_500.py:229-250 does: "
                           "torch RoPE, append, contiguous slice, repeat_interleave, attn_varlen forward"),
        "kernel_only": {"value": round(k_gbs, 2), "unit": "GB/s", "ms_per_sequence": round(k_ms, 3)},
        "e2e": {"value": round(value, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if world > 1:
        line["note"] = f"rank 0 of {world} ran the single-GPU reference; other ranks idle"
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="gqa70b",
                    choices=["gqa70b", "gqa70b_32k", "varlen7b", "mha7b", "prefill16", "llama7b"])
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--gather-ctx", action="store_true",
                    help="kv-head shards: every rank also gets the full ctx of every layer (an unsharded O-proj)")
    ap.add_argument("--gather-impl", choices=["peer", "nccl"], default="peer",
                    help="peer: stores fused into the decode launch over NVLink; nccl: all-gather after it")
    ap.add_argument("--shard-of", type=int, default=1,
                    help="with one GPU: run rank 0's share of an N-way partition of the workload (profiling)")
    ap.add_argument("--no-prefetch-kv", action="store_true",
                    help="decode launches read nothing before the previous launch finishes")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--max-cluster", type=int, default=0,
                    help="largest thread-block cluster of the split decode launch (0 automatic, 1 none)")
    ap.add_argument("--solo-tiles", type=int, default=-1,
                    help="pairs of at most this many tiles are not split in a cluster launch (-1 automatic)")
    ap.add_argument("--stages", type=int, default=0, help="decode pipeline stages per CTA (0 automatic)")
    ap.add_argument("--ctas-per-sm", type=int, default=0, help="decode split-mode CTAs per SM (0 automatic)")
    ap.add_argument("--cluster-min-tiles", type=int, default=0,
                    help="tiles each cluster CTA owns at full arena capacity, at least (0 automatic)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (A/B measurements)")
    ap.add_argument("--kv-len", type=int, default=0, help="decode workloads: every sequence at this many keys")
    ap.add_argument("--no-subrecords", action="store_true",
                    help="skip the per-configuration records (gqa70b_32k, varlen7b, mha7b, prefill16) of the default run")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if (args.max_cluster or args.solo_tiles >= 0 or args.cluster_min_tiles or args.stages or args.ctas_per_sm) \
            and args.impl == "ours":
        import fully_custom_cuda_inference_lamma2_b200 as fcci

        fcci.attn_varlen.set_tuning(stages=args.stages, ctas_per_sm=args.ctas_per_sm, max_cluster=args.max_cluster,
                                    solo_tiles=args.solo_tiles, min_tiles=args.cluster_min_tiles)
    if args.workload == "llama7b":
        (llama_reference if args.impl == "reference" else llama_ours)(args)
    elif args.workload == "prefill16":
        (prefill_reference if args.impl == "reference" else prefill_ours)(args)
    elif args.impl == "reference":
        reference(args)
    else:
        ours(args)


if __name__ == "__main__":
    main()
