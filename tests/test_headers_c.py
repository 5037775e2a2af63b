"""The public headers as a C consumer sees them (CPU only): include/ipuc.h and
include/ipug.h compile as strict C11, and a C program builds a profile report
through ipug_profile_encode that the Python reader decodes field by field."""
import os
import shutil
import subprocess

import pytest

from ipuc import profile as P

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")
LIBDIR = os.path.join(ROOT, "ipu-stack_b200", "ipuc")

pytestmark = pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")


def test_headers_compile_as_c11(tmp_path):
    src = tmp_path / "h.c"
    src.write_text('#include "ipuc.h"\n#include "ipug.h"\nint main(void) { return 0; }\n')
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic", "-fsyntax-only", f"-I{INC}",
                    str(src)], check=True)


def test_c_program_encodes_a_profile(tmp_path):
    exe = tmp_path / "profile_writer"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", f"-I{INC}",
                    os.path.join(ROOT, "tests", "c_consumer", "profile_writer.c"), "-o", str(exe), f"-L{LIBDIR}",
                    "-lipuc", f"-Wl,-rpath,{LIBDIR}"], check=True)
    out = tmp_path / "profile.bin"
    subprocess.run([str(exe), str(out)], check=True)
    rep = P.read(out.read_bytes())
    assert rep.clock_hz == 1_000_000_000
    assert [t.physical_tile for t in rep.tiles] == [3, 4]
    a, b = rep.tiles[0].samples
    assert (a.step.kind, a.step.operation, a.step.kernel, a.start_cycle, a.end_cycle) == (
        "compute", "operation.0", "gemm_f16+gelu", 0, 1000)
    assert a.step.metadata == [("operations", "0,1"), ("tflops", "1450.5")]
    assert (b.step.kind, b.step.kernel, b.step.exchange_event_cycles) == ("exchange", "", 77)
    assert [(x.kind, x.start_cycle, x.end_cycle) for x in b.step.exchange_activities] == [
        ("send", 10, 20), ("partnerBusy", 5, 6)]
    (c,) = rep.tiles[1].samples
    assert (c.step.kind, c.step.operation, c.step.epoch, c.start_cycle, c.end_cycle) == ("idle", "", 2, 7, 9)
