"""The C++ face (include/nmg.hpp) on the device: tests/cpp/nmg_hpp_layer.cpp
drives a Qwen-3.5-shaped per-layer state owner (an attention layer's prefill
and decode step, a delta-rule layer's chunked prefill, clear()) and a Gemma
sliding-window layer; its outputs must match the oracle within the north-star
tolerance (max abs <= 2e-3, rel L2 <= 1e-3)."""
import os
import subprocess

import numpy as np
import pytest

import oracle
from helpers import assert_close, delta_inputs

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = "/usr/local/cuda"
T, HQ, HKV, D, HK, HV, W = 130, 4, 2, 128, 2, 4, 32


def test_cpp_face_runs_a_hybrid_layer_stack(dev, tmp_path):
    exe = tmp_path / "nmg_hpp_layer"
    lib = os.path.join(ROOT, "hero_b200")
    subprocess.run(["g++", "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    "-I", f"{CUDA}/include", os.path.join(ROOT, "tests", "cpp", "nmg_hpp_layer.cpp"), "-L", lib,
                    "-lnmg", f"-Wl,-rpath,{lib}", "-L", f"{CUDA}/lib64", "-lcudart", f"-Wl,-rpath,{CUDA}/lib64",
                    "-o", str(exe)], check=True)
    x = {
        "q": oracle.normal(31, 1, T * HQ * D).reshape(T, HQ * D),
        "k": oracle.normal(31, 2, T * HKV * D).reshape(T, HKV * D),
        "v": oracle.normal(31, 3, T * HKV * D).reshape(T, HKV * D),
        "qd": oracle.normal(31, 4, HQ * D).reshape(1, HQ * D),
        "kd": oracle.normal(31, 5, HKV * D).reshape(1, HKV * D),
        "vd": oracle.normal(31, 6, HKV * D).reshape(1, HKV * D),
        "gq": oracle.normal(31, 7, T * D).reshape(T, D),
        "gk": oracle.normal(31, 8, T * D).reshape(T, D),
        "gv": oracle.normal(31, 9, T * D).reshape(T, D),
    }
    x["dq"], x["dk"], x["dv"], x["g"], x["b"] = delta_inputs(32, T, HK, HV, D)
    for name, a in x.items():
        np.ascontiguousarray(a, dtype=np.float32).tofile(tmp_path / f"{name}.bin")
    r = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout + r.stderr

    got = lambda name, shape: np.fromfile(tmp_path / f"{name}.bin", dtype=np.float32).reshape(shape)
    scale = np.float32(1 / np.sqrt(np.float32(D)))
    want = oracle.attend(x["k"], x["v"], 0, 0, HKV, D, x["q"], HQ, 0, scale=scale)
    assert_close(got("attn", (T, HQ * D)), want, what="attention prefill")
    kk, vv = np.concatenate([x["k"], x["kd"]]), np.concatenate([x["v"], x["vd"]])
    want = oracle.attend(kk, vv, 0, 0, HKV, D, x["qd"], HQ, T, scale=scale)
    assert_close(got("attn_decode", (1, HQ * D)), want, what="attention decode")
    want, ws = oracle.delta_run(np.zeros((HV, D, D), np.float32), x["dq"], x["dk"], x["dv"], x["g"], x["b"], HK)
    assert_close(got("delta", (T, HV, D)), want, what="delta prefill")
    assert_close(got("delta_state", (HV, D, D)), ws, what="delta state")
    # after clear() the same prefill starts from a zero state again
    assert_close(got("delta_again", (T, HV, D)), got("delta", (T, HV, D)), max_abs=1e-5, rel=1e-6,
                 what="delta prefill after clear()")
    want = oracle.attend(x["gk"], x["gv"], 0, W, 1, D, x["gq"], 1, 0, use_scale=False)
    assert_close(got("gemma_local", (T, D)), want, what="gemma sliding window")
