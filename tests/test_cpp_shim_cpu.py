"""The C++ layer (include/bsml_decoder.hpp) compiles against the C ABI, links
libbsml_b200.so and reports the same parameter layout as the Python binding;
without a GPU every failure surfaces as std::runtime_error in the reference's
"brosoundml: <where>: <reason>" format."""

import ctypes
import os
import shutil
import subprocess

import pytest

from brosoundml_b200 import _lib, config

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_shim(tmp_path, gpu=False):
    exe = str(tmp_path / ("shim_gpu" if gpu else "shim_cpu"))
    lib_dir = os.path.join(ROOT, "brosoundml_b200")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", "-I" + os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "cpp", "shim_check.cpp"), "-o", exe, "-L" + lib_dir, "-lbsml_b200",
           "-Wl,-rpath," + lib_dir]
    if gpu:
        cmd[1:1] = ["-DSHIM_GPU", "-I/usr/local/cuda/include"]
        cmd += ["-L/usr/local/cuda/lib64", "-lcudart", "-Wl,-rpath,/usr/local/cuda/lib64"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def write_cfg(tmp_path, cfg):
    c = _lib.make_config(cfg)
    p = tmp_path / "cfg.bin"
    p.write_bytes(ctypes.string_at(ctypes.addressof(c), ctypes.sizeof(c)))
    return str(p)


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_cpp_layer_layout_and_errors(tmp_path):
    exe = build_shim(tmp_path)
    cfg = config.kokoro_82m()
    r = subprocess.run([exe, "layout", write_cfg(tmp_path, cfg)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    n, table, aff_C, _ = _lib.layout(cfg)
    assert f"n_params {n} entries {len(table)} affines {len(aff_C)}" in r.stdout
    assert "block error: brosoundml: bsml_block_create: unknown block kind" in r.stdout
