"""Reader of the per-tensor debug dumps that nnc-py's x86 debug builds and the
cuda target's debug builds write (DEBUG_TENSOR_START <name> <node>, SHAPE,
DIM lines, DATA_START, one value per line, DATA_END, DEBUG_TENSOR_END), the
format nnc-py's own DebugOutputParser reads (tools/debug_compare.py:17-106).
Test infrastructure: the layer-by-layer comparison of the two builds."""

from __future__ import annotations

import numpy as np


def parse(text: str) -> dict[str, dict]:
    """{tensor name: {"node": int, "shape": [...], "data": float32 array}}."""
    out: dict[str, dict] = {}
    cur = None
    vals: list[float] = []
    collecting = False
    for line in text.splitlines():
        line = line.strip()
        if line.startswith("DEBUG_TENSOR_START"):
            _, name, node = line.split()
            cur = {"name": name, "node": int(node), "shape": []}
            collecting = False
        elif cur is None:
            continue
        elif line.startswith("DIM"):
            cur["shape"].append(int(line.split()[2]))
        elif line == "DATA_START":
            collecting, vals = True, []
        elif line == "DATA_END":
            collecting = False
            data = np.array(vals, dtype=np.float32)
            if cur["shape"] and int(np.prod(cur["shape"])) == data.size:
                data = data.reshape(cur["shape"])
            cur["data"] = data
            out[cur["name"]] = cur
            cur = None
        elif collecting and line:
            vals.append(float(line))
    return out


def sample_index(n: int, k: int = 4096) -> np.ndarray:
    """Up to k indices spread evenly over a tensor of n elements."""
    return np.unique(np.linspace(0, n - 1, min(n, k)).round().astype(np.int64))
