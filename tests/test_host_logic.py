"""CPU model of the kernel's work decomposition and of the multi-GPU partitions.

The decode kernel (decode_attn.cu) cuts every (sequence, kv head) pair into
64-key tiles, gives CTA c the tiles [c*N/C, (c+1)*N/C) of the concatenated line,
and stores the partial of pair p computed by CTA c in slot p + c. These tests
restate that arithmetic and check its invariants on random length mixes."""
import random

import pytest

from fully_custom_cuda_inference_lamma2_b200 import sharding

TILE = 64


def tiles_of(L):
    return (L + TILE - 1) // TILE if L > 0 else 1


def cta_of_tile(t, N, C):
    return ((t + 1) * C + N - 1) // N - 1


def decompose(lens, Hkv, C):
    """(pairs, N) where pairs[p] = (first_tile, n_tiles), p = b*Hkv + h."""
    pairs, t = [], 0
    for L in lens:
        n = tiles_of(L)
        for _ in range(Hkv):
            pairs.append((t, n))
            t += n
    return pairs, t


def effective_ctas(lens, Hkv, grid):
    """The kernel's choice of working CTAs C in split mode (decode_attn.cu, after the
    prologue scan): stream-K over min(grid, N), except for uniform lengths, where short
    or numerous pairs get one CTA each, small problems pairs x k CTAs with k dividing a
    pair's tiles, and near-full grids pairs x floor(grid / pairs) CTAs."""
    tiles = [tiles_of(L) * Hkv for L in lens]
    N, P = sum(tiles), len(lens) * Hkv
    C = min(grid, N)
    if len(set(tiles)) == 1 and P <= grid:
        tp = N // P
        if tp <= 8 or (2 * P >= grid and tp <= 32):
            C = P
        elif N < 4 * grid:
            k = min(grid // P, tp)
            while k > 1 and tp % k:
                k -= 1
            C = P * k
        elif 20 * P * (grid // P) >= 17 * grid:
            C = P * (grid // P)
    return C


@pytest.mark.parametrize("seed", range(40))
def test_stream_k_ranges_slots_and_pieces(seed):
    rnd = random.Random(seed)
    B = rnd.randint(1, 70)
    Hkv = rnd.choice([1, 2, 8, 32])
    grid = rnd.choice([1, 7, 148, 296])
    if seed % 2:  # few tiles: fewer than CTAs
        lens = [rnd.choice([0, 1, 15, 64, 65, 200]) for _ in range(rnd.randint(1, 4))]
        B = len(lens)
    else:
        lens = [rnd.choice([0, 1, 15, 64, 65, rnd.randint(1, 40000)]) for _ in range(B)]
    if seed % 4 == 2:  # uniform lengths: the pair-aligned choices
        lens = [rnd.choice([1, 64, 65, 300, 513, 1000, 4097, 20000])] * B
    pairs, N = decompose(lens, Hkv, grid)
    C = effective_ctas(lens, Hkv, grid)  # CTAs past C take no tiles
    assert 1 <= C <= min(grid, N)
    owner = {}
    for c in range(C):
        lo, hi = c * N // C, (c + 1) * N // C
        for t in range(lo, hi):
            assert t not in owner
            owner[t] = c
            assert cta_of_tile(t, N, C) == c
    assert len(owner) == N
    slots = set()
    for p, (first, n) in enumerate(pairs):
        c0, c1 = cta_of_tile(first, N, C), cta_of_tile(first + n - 1, N, C)
        ctas = sorted({owner[t] for t in range(first, first + n)})
        assert ctas == list(range(c0, c1 + 1))  # pieces = c1 - c0 + 1, contiguous
        for c in ctas:
            s = p + c
            assert s not in slots and s < len(pairs) + grid
            slots.add(s)
    if len(set(lens)) == 1 and C != min(grid, N):
        # an aligned choice: no CTA's range holds tiles of two pairs
        pair_of = {}
        for p, (first, n) in enumerate(pairs):
            for t in range(first, first + n):
                pair_of[t] = p
        for c in range(C):
            lo, hi = c * N // C, (c + 1) * N // C
            assert len({pair_of[t] for t in range(lo, hi)}) <= 1


def test_effective_ctas_on_the_measured_shapes():
    assert effective_ctas([4096] * 32, 8, 296) == 256    # 70B shape: one CTA per (sequence, kv head)
    assert effective_ctas([4096] * 32, 1, 296) == 288    # 8-way kv-head shard: 9 CTAs per pair
    assert effective_ctas([513] * 1, 32, 296) == 288     # 1 x 32 heads x 513 keys: 9 tiles per pair, k = 9
    assert effective_ctas([300] * 1, 32, 296) == 32      # short pairs (5 tiles): one CTA each
    assert effective_ctas([1001] * 1, 32, 296) == 256    # 16 tiles per pair, fewer than 4 per CTA: k = 8
    assert effective_ctas([100, 200], 32, 296) == 192    # mixed lengths: stream-K over all 192 tiles
    assert effective_ctas([4096] * 64, 32, 296) == 296   # more pairs than CTAs: stream-K


MAX_CLUSTER = 16  # decode_attn.cu kMaxCluster
SOLO_TILES = 2    # decode_attn.cu kSoloTiles


def cluster_k(P, grid, fits=lambda k: True, max_cluster=MAX_CLUSTER, capacity=None):
    """The host's choice of CTAs per cluster for a split launch (decode_attn.cu,
    launch_decode_t): with at most half as many pairs as resident CTAs, the largest
    k <= min(max_cluster, grid // P, tiles of the arena's capacity) for which P clusters
    of k CTAs are resident at once (`fits`, the occupancy API on the device); 0 = no
    clusters. capacity None stands for the packed layout (no per-sequence bound)."""
    cap_tiles = MAX_CLUSTER if capacity is None else (capacity + TILE - 1) // TILE
    if max_cluster < 2 or 2 * P > grid or cap_tiles < 2:
        return 0
    k = min(max_cluster, grid // P, cap_tiles)
    while k >= 2 and not fits(k):
        k -= 1
    return k if k >= 2 else 0


def cluster_ranges(lens, Hkv, k, solo=SOLO_TILES):
    """Tile ranges of a cluster launch of P*k CTAs with uniform tile counts: CTA
    x = pair*k + r takes part r of k_eff = min(k, tiles per pair) equal parts, or the
    whole pair (k_eff = 1) when it has at most `solo` tiles."""
    pairs, N = decompose(lens, Hkv, 0)
    P = len(pairs)
    tp = N // P
    k_eff = 1 if tp <= solo else min(k, tp)
    out = []
    for x in range(P * k):
        pr, r = divmod(x, k)
        out.append((pr * tp + r * tp // k_eff, pr * tp + (r + 1) * tp // k_eff) if r < k_eff else (0, 0))
    return out, k_eff


def merge_mode(pairs, N, C, p):
    """How pair p's pieces are merged in a launch without clusters (decode_attn.cu,
    segment end): 'whole' (one CTA) or 'single' (the last arriving piece merges all,
    a counter nobody waits on)."""
    first, n = pairs[p]
    c0, c1 = cta_of_tile(first, N, C), cta_of_tile(first + n - 1, N, C)
    return "whole" if c0 == c1 else "single"


def modes(lens, Hkv, grid=296):
    """Merge modes of every pair of a split launch: 'cluster' when the host launches one
    cluster per pair and the lengths give every pair the same tile count (pieces merged
    through distributed shared memory), else those of merge_mode."""
    P = len(lens) * Hkv
    k = cluster_k(P, grid)
    tiles = {tiles_of(L) for L in lens}
    if k and len(tiles) == 1:
        tp = tiles.pop()
        return {"whole" if tp <= SOLO_TILES or min(k, tp) == 1 else "cluster"}
    g = P * k if k else grid
    pairs, N = decompose(lens, Hkv, g)
    C = min(g, N) if k else effective_ctas(lens, Hkv, g)
    return {merge_mode(pairs, N, C, p) for p in range(len(pairs))}


@pytest.mark.parametrize("seed", range(40))
def test_cluster_ranges_cover_each_pair_once(seed):
    rnd = random.Random(2000 + seed)
    Hkv = rnd.choice([1, 2, 4, 8, 32])
    B = rnd.randint(1, 8)
    grid = rnd.choice([148, 296])
    lens = [rnd.choice([0, 1, 63, 64, 65, 513, 4096, 32768, rnd.randint(1, 40000)])] * B
    P = B * Hkv
    k = cluster_k(P, grid)
    if not k:
        assert 2 * P > grid
        return
    assert 2 <= k <= MAX_CLUSTER and P * k <= grid
    ranges, k_eff = cluster_ranges(lens, Hkv, k)
    pairs, N = decompose(lens, Hkv, 0)
    for p, (first, n) in enumerate(pairs):
        got = []
        for r in range(k):
            lo, hi = ranges[p * k + r]
            if r < k_eff:
                assert first <= lo < hi <= first + n  # never empty, never outside the pair
                got.extend(range(lo, hi))
            else:
                assert lo == hi  # idle: joins the cluster barriers only
        assert got == list(range(first, first + n))


@pytest.mark.parametrize("seed", range(40))
def test_cluster_launch_with_mixed_lengths_falls_back_to_stream_k(seed):
    """Mixed tile counts in a cluster launch: stream-K over all P*k CTAs and last-arriver
    merges; the piece slots stay inside the workspace sized for P + grid."""
    rnd = random.Random(3000 + seed)
    Hkv = rnd.choice([1, 2, 8])
    B = rnd.randint(2, 8)
    grid = 296
    lens = [rnd.randint(1, 40000) for _ in range(B)]
    k = cluster_k(B * Hkv, grid)
    if not k:
        return
    g = B * Hkv * k
    pairs, N = decompose(lens, Hkv, g)
    C = min(g, N)
    slots = set()
    for p, (first, n) in enumerate(pairs):
        for c in range(cta_of_tile(first, N, C), cta_of_tile(first + n - 1, N, C) + 1):
            assert p + c < len(pairs) + grid and p + c not in slots
            slots.add(p + c)


def test_merge_modes_on_the_measured_shapes():
    assert modes([4096] * 32, 8) == {"whole"}     # 70B shape on one GPU: one CTA per pair
    assert cluster_k(32, 296) == 9                # 8-way kv-head shard: clusters of 9 CTAs
    assert modes([4096] * 32, 1) == {"cluster"}
    assert cluster_k(64, 296) == 4                # 4-way shard: clusters of 4
    assert modes([4096] * 32, 2) == {"cluster"}
    assert cluster_k(128, 296) == 2               # 2-way shard: pairs of CTAs
    assert modes([4096] * 32, 4) == {"cluster"}
    assert modes([32768] * 4, 8) == {"cluster"}   # 4 x 32k keys: clusters of 9
    assert modes([512 + 1], 32) == {"cluster"}    # config 1 (one sequence, 32 heads): 9 tiles over 9 CTAs
    assert modes([63], 32) == {"whole"}           # one tile per pair: no merge
    assert modes([100], 32) == {"whole"}          # two tiles: one CTA of each cluster carries the pair
    assert "single" in modes([100, 20000], 8) <= {"single", "whole"}  # mixed: stream-K, last arriver
    assert cluster_k(32, 296, fits=lambda k: k <= 8) == 8  # non-portable sizes unavailable
    assert cluster_k(32, 296, capacity=140) == 3           # a short arena bounds the CTAs per pair
    assert cluster_k(32, 296, capacity=64) == 0            # one tile at most: one CTA per pair
    assert cluster_k(32, 296, max_cluster=1) == 0          # clusters turned off


def test_partition_sequences_balances_bytes():
    rnd = random.Random(3)
    lens = [rnd.randint(128, 8192) for _ in range(64)]
    for n in (1, 2, 4, 8):
        parts = sharding.partition_sequences(lens, n)
        assert sorted(i for p in parts for i in p) == list(range(64))
        loads = [sum(lens[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(lens)
        assert parts == sharding.partition_sequences(lens, n)  # deterministic


def test_partition_kv_heads():
    assert sharding.partition_kv_heads(8, 64, 8, 3) == (3, 4, 24, 32)
    assert sharding.partition_kv_heads(8, 64, 2, 1) == (4, 8, 32, 64)
    with pytest.raises(ValueError):
        sharding.partition_kv_heads(8, 64, 3, 0)


def test_partition_by_cost_prefill():
    lens = [256, 4096, 1000, 3000, 500]
    parts = sharding.partition_by_cost([L * (L + 1) / 2 for L in lens], 2)
    assert sorted(i for p in parts for i in p) == list(range(5))
    assert 1 in parts[0]  # the longest goes first to rank 0


def test_bench_algorithmic_work_per_launch():
    """The algorithmic bytes and flops that bench.py divides by the measured launch time:
    K+V of every attended key plus q, ctx and the new rows (decode), and the causal QK^T + PV
    flops (prefill), on the bench workloads and on one rank's share of the 8-way kv-head shards."""
    import bench
    from fully_custom_cuda_inference_lamma2_b200.sharding import partition_kv_heads

    w = bench.workload("gqa70b", None)
    lens1 = [t + 1 for t in w["lens"]]
    assert bench.algorithmic_bytes(w["B"], w["Hq"], w["Hkv"], w["D"], lens1) == 538_312_704
    assert bench.kv_read_bytes(w["Hkv"], w["D"], lens1) == 32 * 4097 * 8 * 128 * 4
    kv_lo, kv_hi, q_lo, q_hi = partition_kv_heads(w["Hkv"], w["Hq"], 8, 0)
    assert (kv_hi - kv_lo, q_hi - q_lo) == (1, 8)
    assert bench.algorithmic_bytes(w["B"], 8, 1, w["D"], lens1) == 67_289_088
    p = bench.prefill_workload("prefill16", None)
    assert sum(p["lens"]) == 39_876
    assert bench.prefill_flops(p["Hq"], p["D"], p["lens"]) == 937_470_803_968


@pytest.mark.parametrize("world", [2, 4, 8])
def test_exchange_slices_tile_every_full_ctx_buffer(world):
    """Each rank's slice of a full-ctx buffer (kv-head partition, slice_offset with the
    decode kernel's out strides [Hq*D, D, 1]) covers its own heads of every sequence;
    together the ranks cover each buffer exactly once, and the flag array, epoch and
    error word sit after the buffers, 256-byte aligned (exchange_layout)."""
    B, Hkv, G, D = 3, 8, 8, 128
    Hq = Hkv * G
    L = sharding.exchange_layout(B, Hq, D, world)
    owner = {}
    for buf in range(L["buffers"]):
        for rank in range(world):
            kv_lo, kv_hi, q_lo, q_hi = sharding.partition_kv_heads(Hkv, Hq, world, rank)
            off = sharding.slice_offset(B, Hq, D, q_lo, buf)
            assert off % 4 == 0
            for b in range(B):
                for h in range(q_hi - q_lo):
                    e0 = off // 2 + b * Hq * D + h * D  # element index in the allocation
                    for e in (e0, e0 + D - 1):
                        assert e not in owner
                        owner[e] = rank
    assert len(owner) == 2 * L["buffers"] * B * Hq
    assert L["flags"] >= L["buffers"] * L["ctx_bytes"] and L["flags"] % 256 == 0
    assert L["epoch"] >= L["flags"] + 4 * world and L["err"] > L["epoch"] and L["total"] > L["err"]
