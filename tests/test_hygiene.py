"""Source checks that keep the library safe to run on shared GPUs (CPU only).

* No batched host/device copy routine of the CUDA runtime or driver: on this
  driver generation they raised GPU faults, so the library issues one
  stream-ordered copy per buffer instead.
* No trap instruction in device code: kernels report failures through the
  device error word and return, so a context stays usable.
* No absolute path of the build machine in the shipped package, the headers,
  the oracle or the benchmark scripts.
"""
import pathlib
import re

ROOT = pathlib.Path(__file__).resolve().parent.parent
PKG = ROOT / "nnc-py_b200"


def _sources(*globs):
    out = []
    for g in globs:
        out += [p for p in ROOT.glob(g) if p.is_file()]
    return out


DEVICE = _sources("nnc-py_b200/csrc/*.cu", "nnc-py_b200/csrc/*.cuh")
HOST = DEVICE + _sources("include/*.h", "oracle/*.c", "oracle/*.py", "nnc-py_b200/nnc_cuda/*.py",
                         "bench.py", "sweep.py", "tests/*.py")


def test_sources_found():
    assert len(DEVICE) >= 8 and len(HOST) > len(DEVICE)


def test_no_batched_copy_routines():
    pat = re.compile(r"Memcpy(?:3D)?BatchAsync")
    hits = [f"{p.relative_to(ROOT)}:{i + 1}" for p in HOST
            for i, line in enumerate(p.read_text(errors="replace").splitlines()) if pat.search(line)]
    assert not hits, hits


def test_no_trap_in_device_code():
    pat = re.compile(r"__trap\s*\(|\"\s*trap\s*;")
    hits = [f"{p.relative_to(ROOT)}:{i + 1}" for p in DEVICE
            for i, line in enumerate(p.read_text(errors="replace").splitlines()) if pat.search(line)]
    assert not hits, hits


def test_no_machine_paths_in_shipped_code():
    pat = re.compile(r"/root/")
    shipped = [p for p in HOST if "tests" not in p.parts]
    hits = [f"{p.relative_to(ROOT)}:{i + 1}" for p in shipped
            for i, line in enumerate(p.read_text(errors="replace").splitlines()) if pat.search(line)]
    assert not hits, hits
