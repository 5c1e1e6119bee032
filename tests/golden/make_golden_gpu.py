"""Writes golden outputs of the reference's own CUDA kernels, run on a B200.

    python tests/golden/make_golden_gpu.py OUT_DIR

Needs oracle/_ref/libref_attn_varlen.so and libref_capture_decode.so (built from the
reference sources by oracle/Makefile). Inputs are regenerated from seeds by
tests/helpers.randn_half; their sha256 is stored so a test can confirm it rebuilt
the same inputs before comparing. Saved as OUT_DIR/ref_kernels.pt; the committed
copy is tests/golden/ref_kernels.pt.
"""
from __future__ import annotations

import math
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from helpers import randn_half, sha256_of  # noqa: E402
import refkernels  # noqa: E402

ATTN_CASES = [  # (H, T, D, seed)
    (32, 1, 128, 1), (32, 2, 128, 2), (32, 63, 128, 3), (32, 64, 128, 4), (32, 65, 128, 5),
    (32, 513, 128, 6), (8, 300, 64, 7), (4, 200, 256, 8), (32, 4097, 128, 9),
]
PLACEHOLDER_CASES = [  # (L, H, max_len, D, vocab, T, ctrl, seed)
    (2, 4, 16, 128, 1000, 5, 1234567, 20), (3, 2, 8, 128, 500, 0, 3, 21), (1, 8, 32, 64, 32000, 31, 31999, 22),
]


def main(out_dir: str):
    dev = "cuda"
    attn = []
    for H, T, D, seed in ATTN_CASES:
        q = randn_half((H, D), 1000 * seed + 1)
        k = randn_half((H, T, D), 1000 * seed + 2)
        v = randn_half((H, T, D), 1000 * seed + 3)
        ctx = refkernels.ref_forward(q.to(dev), k.to(dev), v.to(dev), T, 1.0 / math.sqrt(D))
        torch.cuda.synchronize()
        attn.append({"H": H, "T": T, "D": D, "seed": seed, "scale": 1.0 / math.sqrt(D),
                     "sha_q": sha256_of(q), "sha_k": sha256_of(k), "sha_v": sha256_of(v), "ctx": ctx.cpu()})
    ph = []
    for L, H, max_len, D, vocab, T, ctrl, seed in PLACEHOLDER_CASES:
        ak = randn_half((L, 1, H, max_len, D), 1000 * seed + 1).to(dev)
        av = randn_half((L, 1, H, max_len, D), 1000 * seed + 2).to(dev)
        c = torch.tensor([[ctrl]], dtype=torch.int64, device=dev)
        sl = torch.tensor([T], dtype=torch.int32, device=dev)
        lg = torch.full((1, vocab), 5.0, device=dev)
        refkernels.ref_capture_decode_step(c, ak, av, sl, sl.clone(), lg)
        torch.cuda.synchronize()
        ph.append({"L": L, "H": H, "max_len": max_len, "D": D, "vocab": vocab, "T": T, "ctrl": ctrl, "seed": seed,
                   "sha_k_out": sha256_of(ak), "sha_v_out": sha256_of(av), "logits_nonzero":
                   torch.nonzero(lg[0]).flatten().cpu(), "logits_sum": float(lg.sum()), "seq_len_out": int(sl.item())})
    os.makedirs(out_dir, exist_ok=True)
    path = os.path.join(out_dir, "ref_kernels.pt")
    torch.save({"device": torch.cuda.get_device_name(0), "attn_varlen": attn, "capture_decode": ph}, path)
    print(f"wrote {path}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
