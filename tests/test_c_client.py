"""libqgemm from C: tests/c/qgemm_c_client.c uses nothing but include/qgemm.h, as a
JNI / cgo / ctypes binding does.  It is compiled here with gcc against the in-tree
library; the host-only checks run everywhere, the device checks on a GPU."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c", "qgemm_c_client.c")
LIBDIR = os.path.join(ROOT, "cuda-triton-scala_b200", "lib")


@pytest.fixture(scope="module")
def client(tmp_path_factory):
    import qgemm
    qgemm.lib()  # builds the library if it is missing
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    out = str(tmp_path_factory.mktemp("c_client") / "qgemm_c_client")
    cmd = [gcc, "-O2", "-std=c11", "-Wall", "-Wextra", "-ffp-contract=off",
           "-I", os.path.join(ROOT, "include"), SRC, "-L", LIBDIR, "-lqgemm",
           "-Wl,-rpath," + LIBDIR, "-lm", "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "warning" not in r.stderr, r.stderr
    return out


def test_c_client_host_entry_points(client, tmp_path):
    r = subprocess.run([client, "cpu", str(tmp_path)], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ok" in r.stdout


@pytest.mark.gpu
def test_c_client_device_entry_points(client, tmp_path):
    r = subprocess.run([client, "gpu", str(tmp_path)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ok" in r.stdout
