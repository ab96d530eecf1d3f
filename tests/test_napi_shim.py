"""The N-API shim (nemotron-webgpu-decode_b200/napi/nwd_napi.cc) compiles against the
C ABI header and a stub of the N-API declarations it uses (no Node.js headers in this
image); it binds only functions include/nwd.h declares."""
from __future__ import annotations

import os
import re
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(REPO, "nemotron-webgpu-decode_b200", "napi", "nwd_napi.cc")


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not installed")
def test_shim_compiles(tmp_path):
    # no CUDA include path: the addon reaches the GPU only through include/nwd.h
    cmd = ["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Werror",
           "-I", os.path.join(REPO, "tests", "napi_stub"), "-I", os.path.join(REPO, "include"),
           SHIM]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_shim_calls_only_declared_functions():
    header = open(os.path.join(REPO, "include", "nwd.h")).read()
    declared = set(re.findall(r"\b(nwd_\w+)\s*\(", header))
    used = set(re.findall(r"\b(nwd_\w+)\s*\(", open(SHIM).read()))
    assert used, "the shim binds nothing"
    assert used <= declared, sorted(used - declared)
