"""include/ipuc.h and include/ipug.h from C: programs that link libipuc.so
directly (no Python) build on CPU, and on a GPU runs a GEMM (checked against a host
loop), an attention call and a spec-driven launch, and sees the reference's
validation error for an odd GELU count."""
import os
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
DIR = os.path.join(HERE, "c_consumer")


def build(name="consumer"):
    subprocess.run(["make", "-s", "-C", DIR], check=True, capture_output=True, text=True)
    return os.path.join(DIR, name)


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


def test_c_graph_consumer_plans_without_a_device():
    """include/ipug.h from C: a Repeat over value sequences built with
    ipug_repeat_begin/end, its plan, and rank 1's shard of a 2-GPU split (an
    NCCL all-reduce per block), all on the host."""
    r = subprocess.run([build("graph_consumer"), "--plan-only"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("gemm_f16+gelu") == 2 and "iter=1" in r.stdout
    assert r.stdout.rstrip().endswith("ok")


@pytest.mark.gpu
def test_c_graph_consumer_runs():
    """The same graph run through a session with every value kept, against a
    host evaluation in C with f16 rounding after every op, and the per-op
    diagnostic of the result."""
    r = subprocess.run([build("graph_consumer")], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "diagnose v" in r.stdout and r.stdout.rstrip().endswith("ok")
