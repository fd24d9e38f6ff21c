"""The C++ host side (flour_b200/host/flour_host.h: BlockAllocator, BlockTable, PrefixRegistry,
PagedKvPool, KvCache, Cache, paged_attention, build_batch) through its own test program,
tests/host/test_flour_host.cpp, whose cases follow the reference's unit tests
(src/models/common/paged.rs:288-410, prefix.rs, cache.rs:536-910). Host-only cases run here;
the pool / attention cases run on a GPU and check attention against the C++ oracle."""

import subprocess
from pathlib import Path

import pytest

import oracle
from flour_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "host" / "test_flour_host.cpp"
OUT = ROOT / "tests" / "host" / "_build" / "test_flour_host"


def binary() -> Path:
    deps = [SRC, _lib.LIB_PATH, oracle.LIB_PATH, ROOT / "flour_b200" / "host" / "flour_host.h"]
    if OUT.exists() and all(OUT.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    lib_dir, orc_dir = _lib.LIB_PATH.parent, oracle.LIB_PATH.parent
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-I", str(ROOT / "include"),
           "-I", str(ROOT / "flour_b200" / "host"), str(SRC), "-o", str(OUT),
           "-L", str(lib_dir), "-lflour_attn", f"-Wl,-rpath,{lib_dir}",
           "-L", str(orc_dir), "-l:liboracle.so", f"-Wl,-rpath,{orc_dir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return OUT


def run(*args):
    r = subprocess.run([str(binary()), *args], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_host_logic_matches_reference_tests():
    out = run()
    assert "0 failed" in out and "FAIL" not in out, out


@pytest.mark.gpu
def test_host_pool_and_attention_on_gpu():
    out = run("--gpu")
    assert "0 failed" in out and "FAIL" not in out, out
    assert "attention_matches_oracle" in out
