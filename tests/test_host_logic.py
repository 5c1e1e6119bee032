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


COOP_PIECES = 6  # decode_attn.cu kCoopPieces


def merge_mode(pairs, N, C, p):
    """How pair p's pieces are merged (decode_attn.cu, segment end): 'whole' (one CTA),
    'slices' (every piece ends its CTA's range and there are at least COOP_PIECES pieces:
    the piece CTAs wait for one another and merge a slice each) or 'single' (the last
    arriving piece merges all)."""
    first, n = pairs[p]
    c0, c1 = cta_of_tile(first, N, C), cta_of_tile(first + n - 1, N, C)
    if c0 == c1:
        return "whole"
    if c1 - c0 + 1 >= COOP_PIECES and first + n == (c1 + 1) * N // C:
        return "slices"
    return "single"


@pytest.mark.parametrize("seed", range(40))
def test_slice_merge_never_holds_up_a_later_segment(seed):
    rnd = random.Random(1000 + seed)
    Hkv = rnd.choice([1, 2, 8, 32])
    grid = rnd.choice([148, 296])
    B = rnd.randint(1, 40)
    lens = [rnd.choice([4096, 1000, 513, rnd.randint(1, 40000)])] * B if seed % 2 else \
        [rnd.randint(1, 40000) for _ in range(B)]
    pairs, N = decompose(lens, Hkv, grid)
    C = effective_ctas(lens, Hkv, grid)
    for p, (first, n) in enumerate(pairs):
        if merge_mode(pairs, N, C, p) != "slices":
            continue
        # every piece CTA's range ends inside this pair: waiting there delays nothing else
        for c in range(cta_of_tile(first, N, C), cta_of_tile(first + n - 1, N, C) + 1):
            assert first < (c + 1) * N // C <= first + n


def test_merge_modes_on_the_measured_shapes():
    def modes(lens, Hkv, grid=296):
        pairs, N = decompose(lens, Hkv, grid)
        C = effective_ctas(lens, Hkv, grid)
        return {merge_mode(pairs, N, C, p) for p in range(len(pairs))}
    assert modes([4096] * 32, 8) == {"whole"}     # 70B shape on one GPU: one CTA per pair
    assert modes([4096] * 32, 1) == {"slices"}    # 8-way kv-head shard: 9 pieces per pair
    assert modes([4096] * 32, 2) == {"single"}    # 4-way shard: 4 pieces per pair
    assert modes([4096] * 32, 4) == {"single"}    # 2-way shard: 2 pieces per pair
    assert modes([32768] * 4, 8) == {"slices"}    # 4 x 32k keys
    assert modes([1001], 32) == {"slices"}        # 1 x 32 heads x 1001 keys: 8 pieces per pair


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
