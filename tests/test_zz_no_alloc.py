"""The allocation-free entry point, checked through the C ABI against the
regular one.

fcci_decode_attention_noalloc serves callers that may not allocate device
memory (a host runtime that owns the whole device pool, or an FFI with no way
to reach an allocator): they pass inputs and outputs only, and the split-KV
scratch comes from a fixed array inside the library. Its results must match
fcci_decode_attention given a caller-allocated workspace, within the tolerance
of the other decode tests, on consecutive calls that reuse that array.

The file name sorts last so that a run stopping at the first failure has run
every other test first; the test also passes alone in a fresh process.
"""
import ctypes

import pytest
import torch

import capi_ctypes as C
from helpers import randn_half
from oracle import decode_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _lib():
    lib = C.load()
    # a void* descriptor argument, so that version-1 descriptors (no trailing flags) pass too
    lib.fcci_decode_attention_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    lib.fcci_decode_attention_noalloc.restype = ctypes.c_int
    lib.fcci_decode_noalloc_read_error.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int, ctypes.c_void_p]
    lib.fcci_decode_noalloc_read_error.restype = ctypes.c_int
    return lib


def _as_v1(d):
    """The same descriptor in the version-1 layout, which ends before `flags`."""
    v1 = C.DecodeDescV1()
    ctypes.memmove(ctypes.addressof(v1), ctypes.addressof(d), ctypes.sizeof(v1))
    v1.abi_version = 1
    return v1


def _noalloc_error(lib):
    flags = ctypes.c_uint32(0)
    rc = lib.fcci_decode_noalloc_read_error(ctypes.byref(flags), 1, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.fcci_last_error_string()
    return flags.value


def _case(B, Hkv, G, D, lens, cap, seed):
    q = randn_half((B, Hkv * G, D), seed)
    kn, vn = randn_half((B, Hkv, D), seed + 1), randn_half((B, Hkv, D), seed + 2)
    kc, vc = randn_half((B, Hkv, cap, D), seed + 3), randn_half((B, Hkv, cap, D), seed + 4)
    return q, kn, vn, kc, vc, torch.tensor(lens, dtype=torch.int32)


def _run(lib, entry, case, split, workspace=None, flags=0, v1=False):
    """One decode step (RoPE + append + attention + advance) on fresh device copies."""
    q, kn, vn, kc, vc, T = case
    dq, dkn, dvn, dk, dv, dT = (t.to(DEV) for t in (q, kn, vn, kc, vc, T))
    out = torch.empty_like(dq)
    d = C.batched_desc(dq, dk, dv, out, k_new=dkn, v_new=dvn, seq_lens=dT, advance=True, split=split,
                       workspace=workspace, flags=flags)
    if v1:
        d = _as_v1(d)
    rc = entry(ctypes.addressof(d), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, lib.fcci_last_error_string()
    return out.cpu(), dk.cpu(), dT.cpu()


def test_noalloc_matches_workspace_entry_on_consecutive_calls():
    lib = _lib()
    lib.fcci_decode_attention.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    cases = [  # different shapes back to back, so each call reuses the array
        (_case(3, 4, 8, 128, [5, 300, 640], 700, 10), True),
        (_case(5, 2, 1, 128, [0, 63, 64, 1000, 2047], 2048, 20), True),
    ]
    for i, (case, split) in enumerate(cases):
        q, kn, vn, kc, vc, T = case
        B, Hq, D = q.shape
        Hkv = kn.shape[1]
        nbytes = lib.fcci_decode_workspace_bytes(B, Hq, Hkv, D, torch.cuda.current_device())
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
        ref_out, ref_k, ref_T = _run(lib, lib.fcci_decode_attention, case, split, ws)
        na_out, na_k, na_T = _run(lib, lib.fcci_decode_attention_noalloc, case, split)
        max_abs, rel = O.compare(na_out.float(), ref_out.float())
        assert max_abs <= O.MAX_ABS_TOL and rel <= O.REL_L2_TOL, f"call {i}: max_abs={max_abs} rel={rel}"
        assert torch.equal(na_k, ref_k), f"call {i}: appended rows differ"
        assert na_T.tolist() == ref_T.tolist() == [t + 1 for t in T.tolist()]
        want = O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn)
        max_abs, rel = O.compare(na_out.float(), want["ctx"])
        assert max_abs <= O.MAX_ABS_TOL and rel <= O.REL_L2_TOL, f"call {i} vs oracle: {max_abs} {rel}"
        assert _noalloc_error(lib) == 0


@pytest.mark.parametrize("variant", ["abi_v1", "prefetch_kv"])
def test_noalloc_descriptor_variants_match_workspace_entry(variant):
    """A version-1 descriptor (no flags field) and FCCI_DECODE_PREFETCH_KV through the
    allocation-free entry point give what the workspace entry point gives."""
    lib = _lib()
    lib.fcci_decode_attention.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    case = _case(4, 8, 8, 128, [4095, 17, 2048, 600], 4100, 30)
    q, kn, vn, kc, vc, T = case
    B, Hq, D = q.shape
    nbytes = lib.fcci_decode_workspace_bytes(B, Hq, kn.shape[1], D, torch.cuda.current_device())
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    flags = C.PREFETCH_KV if variant == "prefetch_kv" else 0
    v1 = variant == "abi_v1"
    ref_out, ref_k, ref_T = _run(lib, lib.fcci_decode_attention, case, True, ws, flags=flags, v1=v1)
    for _ in range(2):  # two calls in a row on the shared array
        na_out, na_k, na_T = _run(lib, lib.fcci_decode_attention_noalloc, case, True, flags=flags, v1=v1)
        assert torch.equal(na_out, ref_out), variant
        assert torch.equal(na_k, ref_k) and na_T.tolist() == ref_T.tolist()
        assert _noalloc_error(lib) == 0
    want = O.decode_step(q, kc, vc, T, k_new=kn, v_new=vn)
    max_abs, rel = O.compare(na_out.float(), want["ctx"])
    assert max_abs <= O.MAX_ABS_TOL and rel <= O.REL_L2_TOL, f"{variant} vs oracle: {max_abs} {rel}"


def test_noalloc_reports_capacity_overflow():
    """A sequence whose T + 1 exceeds the arena capacity sets FCCI_DEV_ERR_CAPACITY in the
    built-in scratch's error word; the caller reads it with fcci_decode_noalloc_read_error."""
    lib = _lib()
    case = _case(3, 2, 4, 128, [10, 400, 20], 400, 40)
    out, _, T = _run(lib, lib.fcci_decode_attention_noalloc, case, True)
    assert _noalloc_error(lib) & 1
    assert torch.count_nonzero(out[1]) == 0
    assert T.tolist() == [11, 400, 21]
    assert _noalloc_error(lib) == 0  # cleared by the read above


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _lib()
    B, Hkv, G, D = 4096, 8, 8, 128  # ~4096*8 pieces of 4 KB: far beyond the fixed scratch
    q = torch.zeros(B, Hkv * G, D, dtype=torch.float16, device=DEV)
    kc = torch.zeros(1, Hkv, 16, D, dtype=torch.float16, device=DEV).expand(B, Hkv, 16, D)
    d = C.batched_desc(q, kc, kc, q, fixed_len=4, split=True)
    assert lib.fcci_decode_attention_noalloc(ctypes.addressof(d), None) == 3
    assert b"scratch" in lib.fcci_last_error_string()
