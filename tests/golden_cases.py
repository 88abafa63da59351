"""Loads the committed golden fixtures (tests/golden/cases.json + golden.npz)."""

from __future__ import annotations

import functools
import json
import pathlib

import numpy as np

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


@functools.lru_cache(maxsize=1)
def _load():
    cases = json.loads((GOLDEN / "cases.json").read_text())
    blobs = np.load(GOLDEN / "golden.npz")
    return cases, {k: blobs[k] for k in blobs.files}


def cases():
    return _load()[0]


def inputs(case):
    blobs = _load()[1]
    pre = f"{case['name']}/in/"
    return {k[len(pre):]: v for k, v in blobs.items() if k.startswith(pre)}


def outputs(case):
    blobs = _load()[1]
    pre = f"{case['name']}/out/"
    return {k[len(pre):]: v for k, v in blobs.items() if k.startswith(pre)}


def names():
    return [c["name"] for c in cases()]


def by_name(name):
    for c in cases():
        if c["name"] == name:
            return c
    raise KeyError(name)
