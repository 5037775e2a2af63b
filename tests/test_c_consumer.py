"""include/ipuc.h from C: a program that links libipuc.so directly (no
Python) builds on CPU, and on a GPU runs a GEMM (checked against a host
loop), an attention call and a spec-driven launch, and sees the reference's
validation error for an odd GELU count."""
import os
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
DIR = os.path.join(HERE, "c_consumer")


def build():
    subprocess.run(["make", "-s", "-C", DIR], check=True, capture_output=True, text=True)
    return os.path.join(DIR, "consumer")


def test_c_consumer_builds_against_header_and_library():
    exe = build()
    assert os.access(exe, os.X_OK)


@pytest.mark.gpu
def test_c_consumer_runs():
    exe = build()
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "spec gemm -> ipuc_gemm_f16 (replaces ipu_stack_gemm_f16_init)" in r.stdout
    assert "odd GELU: IPUC_ERR_INVALID_ARGUMENT: kernel ipu_stack_gelu_tanh_approx_f16 requires an element count " \
           "divisible by 2, got 7" in r.stdout
    assert r.stdout.rstrip().endswith("ok")
