#!/usr/bin/env python3
"""Generate the committed golden fixtures from the reference's own torch restatements.

The reference ships pure-torch restatements of its sparse ops, ``tools/ref_sparse_conv.py``
and ``tools/ref_c2s.py``. They load checkpoint weights from a path that does not exist
here, so this script does not import them as modules. It parses each file and executes
the reference's own statements and functions: the seeded input generators, the neighbor
table loop, ``submconv``, ``nbr_table`` and the C2S block. It supplies seeded random
weights in place of the checkpoint load and skips the ``np.save`` / ``os.makedirs``
statements. What it writes:

* ``submconv_ref.npz``: ``tools/ref_sparse_conv.py:38-80``. R=16, N=800, seed 3. It holds
  the reference's neighbor table [N,27] (-1 = absent), conv_out and the ConvNeXt
  block_out, at C=32 with random weights.
* ``c2s_ref.npz``: ``tools/ref_c2s.py:30-79``. R=16, N=600, seed 5, Cin=32, Cout=16. It
  holds subdiv logits, the mask, new_coords, the (parent, octant) gather list and out.
* ``nbr_cases.npz``: the reference's ``nbr_table`` (``tools/ref_c2s.py:38-48``) on edge
  cases: duplicate coordinates (last writer wins), coordinates at 0 whose neighbors are
  negative, a dense 3^3 block, an isolated voxel, and one voxel.

Weights are drawn as bf16-representable float32 values, so the same fixture also serves
the bf16 operand mode exactly. Run it where the reference project is present, at
``$TRELLIS_REF`` (default: a ``reference`` directory beside this repository). The GPU box
never runs it: tests read only the .npz files.
"""
from __future__ import annotations

import ast
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("TRELLIS_REF", os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))), "reference"))


def _bf16_exact(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def _rand_w(shape, fan_in, seed):
    g = torch.Generator().manual_seed(seed)
    return _bf16_exact(torch.randn(*shape, generator=g) / float(np.sqrt(fan_in)))


def _is_skipped(node: ast.stmt) -> bool:
    """Statements of the reference scripts that touch the filesystem or the checkpoint."""
    src = ast.unparse(node)
    if isinstance(node, ast.Assign):
        names = [t.id for t in node.targets if isinstance(t, ast.Name)]
        if any(n in ("CK", "OUT", "w") for n in names):
            return True
    if "np.save" in src or "os.makedirs" in src or "OUT" in src:
        return True
    return False


def _exec_reference(path: str, ns: dict, stop_after_line: int | None = None) -> dict:
    """Execute the top-level statements of a reference script in ``ns`` (skipping I/O)."""
    tree = ast.parse(open(path).read(), filename=path)
    for node in tree.body:
        if stop_after_line is not None and node.lineno > stop_after_line:
            break
        if _is_skipped(node):
            continue
        code = compile(ast.Module(body=[node], type_ignores=[]), path, "exec")
        exec(code, ns)
    return ns


def make_submconv(C: int = 32) -> dict:
    blk = "blocks.3.0"
    w = {
        f"{blk}.conv.weight": _rand_w((C, 3, 3, 3, C), 27 * C, 101),
        f"{blk}.conv.bias": _rand_w((C,), 100, 102),
        f"{blk}.norm.weight": 1.0 + _rand_w((C,), 100, 103),
        f"{blk}.norm.bias": _rand_w((C,), 100, 104),
        f"{blk}.mlp.0.weight": _rand_w((4 * C, C), C, 105),
        f"{blk}.mlp.0.bias": _rand_w((4 * C,), 100, 106),
        f"{blk}.mlp.2.weight": _rand_w((C, 4 * C), 4 * C, 107),
        f"{blk}.mlp.2.bias": _rand_w((C,), 100, 108),
    }
    ns = {"__name__": "ref_sparse_conv", "w": w}
    _exec_reference(os.path.join(REF, "tools/ref_sparse_conv.py"), ns)
    out = {
        "coords": ns["coords"].numpy().astype(np.int32),
        "feats": ns["feats"].numpy().astype(np.float32),
        "nbr_ref": ns["nbr"].numpy().astype(np.int32),            # [N,27], -1 = absent
        "weight": w[f"{blk}.conv.weight"].numpy(),                 # [Co,3,3,3,Ci]
        "bias": w[f"{blk}.conv.bias"].numpy(),
        "conv_out": ns["conv_out"].numpy().astype(np.float32),
        "block_out": ns["block_out"].numpy().astype(np.float32),
    }
    for k in ("norm.weight", "norm.bias", "mlp.0.weight", "mlp.0.bias", "mlp.2.weight", "mlp.2.bias"):
        out[k] = w[f"{blk}.{k}"].numpy()
    return out


def make_c2s(Cin: int = 32, Cout: int = 16) -> dict:
    P = "blocks.3.4"
    w = {
        f"{P}.conv1.weight": _rand_w((Cout * 8, 3, 3, 3, Cin), 27 * Cin, 201),
        f"{P}.conv1.bias": _rand_w((Cout * 8,), 100, 202),
        f"{P}.conv2.weight": _rand_w((Cout, 3, 3, 3, Cout), 27 * Cout, 203),
        f"{P}.conv2.bias": _rand_w((Cout,), 100, 204),
        f"{P}.norm1.weight": 1.0 + _rand_w((Cin,), 100, 205),
        f"{P}.norm1.bias": _rand_w((Cin,), 100, 206),
        f"{P}.to_subdiv.weight": _rand_w((8, Cin), Cin, 207),
        f"{P}.to_subdiv.bias": _rand_w((8,), 100, 208),
    }
    ns = {"__name__": "ref_c2s", "w": w}
    _exec_reference(os.path.join(REF, "tools/ref_c2s.py"), ns)
    gl = np.array(ns["gidx"], dtype=np.int32).reshape(-1, 2)      # (parent i, octant o)
    out = {
        "coords": ns["coords"].numpy().astype(np.int32),
        "feats": ns["feats"].numpy().astype(np.float32),
        "subdiv": ns["subdiv"].numpy().astype(np.float32),        # logits [N,8]
        "mask": ns["mask"].numpy().astype(np.uint8),              # [N,8]
        "new_coords": ns["new_coords_t"].numpy().astype(np.int32),
        "gather_parent": gl[:, 0].copy(),
        "gather_octant": gl[:, 1].copy(),
        "out": ns["out"].numpy().astype(np.float32),
    }
    for k in ("conv1.weight", "conv1.bias", "conv2.weight", "conv2.bias", "norm1.weight",
              "norm1.bias", "to_subdiv.weight", "to_subdiv.bias"):
        out[k] = w[f"{P}.{k}"].numpy()
    # the same script's nbr_table, kept for the edge cases below
    return out, ns["nbr_table"]


def make_nbr_cases(nbr_table) -> dict:
    cases = {}
    rng = np.random.default_rng(11)
    base = rng.integers(0, 6, size=(60, 3))
    dup = np.concatenate([base, base[rng.integers(0, 60, 25)]], 0)   # 25 duplicated rows
    rng.shuffle(dup)
    cases["dups"] = dup
    cases["origin_corner"] = np.array([[0, 0, 0], [1, 0, 0], [0, 1, 0], [0, 0, 1], [1, 1, 1]])
    cases["dense3"] = np.stack(np.meshgrid(np.arange(3), np.arange(3), np.arange(3),
                                           indexing="ij"), -1).reshape(-1, 3)
    cases["isolated"] = np.array([[5, 5, 5], [9, 9, 9]])
    cases["single"] = np.array([[7, 3, 1]])
    cases["far"] = np.array([[1023, 1023, 1023], [1022, 1023, 1023], [0, 512, 1023]])
    out = {}
    for name, c in cases.items():
        ct = torch.tensor(c, dtype=torch.int64)
        out[f"{name}_coords"] = c.astype(np.int32)
        out[f"{name}_nbr"] = nbr_table(ct).numpy().astype(np.int32)
    return out


def main() -> int:
    if not os.path.isdir(os.path.join(REF, "tools")):
        print(f"reference not found at {REF}", file=sys.stderr)
        return 1
    torch.manual_seed(0)
    sc = make_submconv()
    np.savez_compressed(os.path.join(HERE, "submconv_ref.npz"), **sc)
    c2s, nbr_table = make_c2s()
    np.savez_compressed(os.path.join(HERE, "c2s_ref.npz"), **c2s)
    np.savez_compressed(os.path.join(HERE, "nbr_cases.npz"), **make_nbr_cases(nbr_table))
    for f in ("submconv_ref.npz", "c2s_ref.npz", "nbr_cases.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")
    return 0


if __name__ == "__main__":
    sys.exit(main())
