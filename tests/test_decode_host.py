"""The device decoder of Q2_K, Q3_K and Q8_0 (kernite_b200/csrc/kq_decode.cuh, __host__
__device__ functions) compiled for the host and checked without a GPU: bit for bit against the
gguf-py 0.19.0 fixtures and the CPU oracle. The GPU tests then check the kernel that calls the
same functions (tests/test_more_types_gpu.py)."""
import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TYPES = [2, 3, 8]


@pytest.fixture(scope="module")
def host(tmp_path_factory):
    nvcc = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc) and not shutil.which(nvcc):
        pytest.skip("nvcc not found")
    out = str(tmp_path_factory.mktemp("kqh") / "libkqh.so")
    subprocess.run([nvcc, "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-Xcompiler", "-fPIC,-ffp-contract=off", "-shared",
                    "-I", os.path.join(ROOT, "kernite_b200", "csrc"), "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "host", "host_decode.cu"), "-o", out], check=True)
    L = ctypes.CDLL(out)
    L.kqh_dequant.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
    return L


def dequant(L, qtype, blocks):
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    n = blocks.size // oracle.block_bytes(qtype)
    out = np.empty(n * 256, dtype=np.float32)
    assert L.kqh_dequant(qtype, blocks.ctypes.data, n, out.ctypes.data) == 0
    return out


@pytest.mark.parametrize("qtype", TYPES)
@pytest.mark.parametrize("which", ["gen", "raw", "kat"])
def test_device_decode_source_matches_gguf(host, golden, qtype, which):
    pre = oracle.GOLDEN_PREFIX[qtype]
    want = golden[f"{pre}_{which}_f32bits"]
    got = dequant(host, qtype, golden[f"{pre}_{which}_blocks"]).view(np.uint32)
    nan = np.isnan(want.view(np.float32))
    assert np.array_equal(np.isnan(got.view(np.float32)), nan)
    assert np.array_equal(got[~nan], want[~nan])


@pytest.mark.parametrize("qtype", TYPES)
def test_device_decode_source_matches_oracle_on_generated(host, qtype):
    blocks = oracle.fill(qtype, oracle.stream_key(11, qtype), 123, 500)
    assert np.array_equal(dequant(host, qtype, blocks).view(np.uint32),
                          oracle.dequant(qtype, blocks).view(np.uint32))
