"""CPU checks of the native boundary: the C-ABI library loads and exports every
function declared in include/*.h; the pybind modules carry the reference's names."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "fully_custom_cuda_inference_lamma2_b200", "libfcci_decode.so")


def declared_functions():
    names = []
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not h.endswith(".h"):
            continue
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", src, flags=re.M):
            name = m.group(1)
            if name not in ("if", "defined", "sizeof"):
                names.append(name)
    return sorted(set(names))


def test_headers_declare_the_reference_symbols():
    names = declared_functions()
    for sym in ("attn_varlen_host", "capture_decode_host", "capture_decode_host_ext", "rmsnorm_host",
                "swiglu_host", "prepare_cublas_handle", "fcci_decode_attention", "fcci_rope_append"):
        assert sym in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_library_status_calls_without_gpu():
    lib = ctypes.CDLL(LIB)
    lib.fcci_last_status.restype = ctypes.c_int
    lib.fcci_decode_workspace_bytes.restype = ctypes.c_size_t
    lib.fcci_decode_workspace_bytes.argtypes = [ctypes.c_int32] * 4 + [ctypes.c_int]
    lib.fcci_decode_attention.restype = ctypes.c_int
    lib.fcci_decode_attention.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    lib.fcci_launch_count.restype = ctypes.c_uint64
    # invalid shapes are rejected before any device query
    assert lib.fcci_decode_workspace_bytes(0, 8, 8, 128, 0) == 0
    assert lib.fcci_decode_workspace_bytes(2, 6, 4, 128, 0) == 0
    # a null descriptor is an argument error, not a crash
    assert lib.fcci_decode_attention(None, None) == 1
    assert lib.fcci_launch_count() == 0


def test_pybind_modules_mirror_the_reference_surface():
    import fully_custom_cuda_inference_lamma2_b200 as pkg

    av, cds = pkg.attn_varlen, pkg.capture_decode_step
    assert av.__name__.split(".")[-1] == "attn_varlen" and cds.__name__.split(".")[-1] == "capture_decode_step"
    # custom_kernels/attn_varlen.cpp:47-49 and capture_decode_step.cpp:312-325
    assert callable(av.forward)
    for f in ("capture_decode", "capture_decode_ext", "prepare_cublas", "rmsnorm", "rmsnorm_ptr", "swiglu",
              "gate_up_gemm", "down_gemm", "logits_gemm_vocab"):
        assert callable(getattr(cds, f)), f
    doc = av.forward.__doc__
    assert re.search(r"forward\(q: torch\.Tensor, k: torch\.Tensor, v: torch\.Tensor, seq_len: \S*Int\S*, "
                     r"scale: \S*Float\S*\) -> torch\.Tensor", doc), doc


def test_dropin_import_by_name():
    import importlib
    import sys

    import fully_custom_cuda_inference_lamma2_b200 as pkg

    sys.path.insert(0, pkg.dropin_path())
    try:
        m = importlib.import_module("capture_decode_step")
        assert hasattr(m, "capture_decode")
    finally:
        sys.path.remove(pkg.dropin_path())


def test_forward_checks_run_on_host():
    import torch

    import fully_custom_cuda_inference_lamma2_b200 as pkg

    q = torch.zeros(4, 128, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="must be CUDA"):
        pkg.attn_varlen.forward(q, q.view(4, 1, 128), q.view(4, 1, 128), 1, 1.0)


def test_descriptor_layout_matches_header(tmp_path):
    """The ctypes descriptors (version 2, and version 1 without the trailing flags) have
    the C header's size and field offsets."""
    import subprocess

    import capi_ctypes as C

    src = tmp_path / "layout.cpp"
    src.write_text(
        '#include <cstdio>\n#include <cstddef>\n#include "fcci_decode.h"\n'
        "int main() { std::printf(\"%zu %zu %zu %d %u\\n\", sizeof(fcci_decode_desc),"
        " offsetof(fcci_decode_desc, workspace_bytes), offsetof(fcci_decode_desc, flags),"
        " FCCI_DECODE_ABI_VERSION, FCCI_DECODE_PREFETCH_KV); return 0; }\n")
    exe = tmp_path / "layout"
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    subprocess.run(["g++", "-I", os.path.join(ROOT, "include"), "-I", cuda_inc, str(src), "-o", str(exe)],
                   check=True)
    size, off_wsb, off_flags, abi, prefetch = subprocess.run([str(exe)], check=True, capture_output=True,
                                                             text=True).stdout.split()
    assert int(size) == ctypes.sizeof(C.DecodeDesc)
    assert int(off_flags) == C.DecodeDesc.flags.offset
    assert int(off_wsb) == C.DecodeDesc.workspace_bytes.offset == C.DecodeDescV1.workspace_bytes.offset
    assert ctypes.sizeof(C.DecodeDescV1) <= int(off_flags)
    assert int(abi) == C.ABI_VERSION and int(prefetch) == C.PREFETCH_KV
