"""The MpsContext adapter (kraken-infer_b200/adapter/mps_context_kib.cpp):
compiled against the reference's own, unchanged mps_backend.hpp and linked to
libkib.so, it is the drop-in a kraken-infer build links in place of
mps_backend.mm.  Without a B200 its create() reports unavailable, as the
reference's stub does; on a B200 it runs ops through the reference's member
signatures and checks them."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ADAPTER = os.path.join(ROOT, "kraken-infer_b200", "adapter")
EXE = os.path.join(ADAPTER, "_build", "kib_adapter_check")
REF = os.environ.get("KIB_REFERENCE_ROOT", os.path.join(os.path.dirname(ROOT), "reference"))


def _build():
    if os.path.isdir(os.path.join(REF, "include", "toyllm")):
        subprocess.check_call(["make", "-s", "-C", ADAPTER, "REF_ROOT=" + REF])
    if not os.path.exists(EXE):
        pytest.skip("the adapter needs the reference's headers to build (not present on this machine)")


def test_adapter_builds_and_reports_unavailable_without_a_b200():
    _build()
    import conftest
    out = subprocess.run([EXE], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    if conftest.gpu_available():
        assert out.stdout.strip() == "ok", out.stdout
    else:
        assert out.stdout.startswith("unavailable"), out.stdout


@pytest.mark.gpu
def test_adapter_runs_ops_on_the_gpu():
    _build()
    out = subprocess.run([EXE], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.strip() == "ok", out.stdout + out.stderr
