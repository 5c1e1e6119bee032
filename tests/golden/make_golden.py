"""Writes tests/golden/rope_reference.pt from the reference's own RoPE code.

Run where the reference checkout exists (REF env var, default /root/reference):

    python tests/golden/make_golden.py

Two reference functions are lifted verbatim out of their source files with `ast`
and executed unchanged on the CPU:
  * `apply_rope_` — nested in main() of scripts/direct_custom_decode_500.py
    (lines 90-108): the decode driver's RoPE, fp32 math rounded to fp16.
  * `_init_rope_cache` + `_apply_rope_inplace_heads` — methods of GraphGenerator in
    case4_graph_generator_server_ipc.py (lines 869-898): the server's table-based
    RoPE, applied to fp32 heads.
Inputs are seeded fp16 N(0,1) rows; positions cover 0, small, tile-edge and long
contexts, rotary_dim 128 (full) and 64 (partial, driver only), theta 1e4 and 5e5.
"""
from __future__ import annotations

import ast
import os
import sys
import types

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("REF", "/root/reference")
POSITIONS = [0, 1, 7, 63, 64, 511, 512, 4095, 4096, 32767, 32768]


def lift_function(path: str, name: str):
    """Source of the (possibly nested) function `name` in `path`, dedented, as a code string."""
    src = open(path).read()
    tree = ast.parse(src)
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and node.name == name:
            seg = ast.get_source_segment(src, node)
            lines = seg.splitlines()
            indent = len(lines[0]) - len(lines[0].lstrip())
            # decorators are not part of the segment; staticmethod is dropped on purpose
            return "\n".join(l[indent:] if len(l) >= indent else l for l in lines)
    raise KeyError(f"{name} not found in {path}")


def main():
    drv = os.path.join(REF, "scripts", "direct_custom_decode_500.py")
    srv = os.path.join(REF, "case4_graph_generator_server_ipc.py")
    ns: dict = {"torch": torch}
    exec(compile(lift_function(drv, "apply_rope_"), drv, "exec"), ns)
    exec(compile(lift_function(srv, "_init_rope_cache"), srv, "exec"), ns)
    exec(compile(lift_function(srv, "_apply_rope_inplace_heads"), srv, "exec"), ns)
    apply_rope_ = ns["apply_rope_"]
    init_cache = ns["_init_rope_cache"]
    apply_heads = ns["_apply_rope_inplace_heads"]

    g = torch.Generator().manual_seed(2024)
    n_heads, D = 8, 128
    cases = []
    for theta in (10000.0, 500000.0):
        for rot in (128, 64):
            for pos in POSITIONS:
                x = torch.randn(n_heads, D, generator=g).half()
                out = apply_rope_(x.clone(), pos, rot, theta, torch.device("cpu"))
                cases.append({"kind": "driver", "theta": theta, "rotary_dim": rot, "pos": pos, "x": x,
                              "out": out.clone()})
        # server variant: full rotary over head_dim, fp32 heads
        fake = types.SimpleNamespace(
            device=torch.device("cpu"), hidden_size=n_heads * D, num_heads_cfg=n_heads,
            model=types.SimpleNamespace(config=types.SimpleNamespace(rope_theta=theta)))
        init_cache(fake, max_len=max(POSITIONS) + 1)
        for pos in POSITIONS:
            x = torch.randn(n_heads, D, generator=g).half()
            h = x.float().clone()
            apply_heads(h, fake.rope_cos, fake.rope_sin, pos)
            cases.append({"kind": "server", "theta": theta, "rotary_dim": D, "pos": pos, "x": x, "out": h.clone()})
    out = os.path.join(HERE, "rope_reference.pt")
    torch.save({"source": {"driver": "scripts/direct_custom_decode_500.py:90-108",
                           "server": "case4_graph_generator_server_ipc.py:869-898"},
                "cases": cases}, out)
    print(f"wrote {len(cases)} cases to {out}")


if __name__ == "__main__":
    sys.exit(main())
