"""The C++ host API (include/rustane.hpp) through its own C++ test program
(tests/cpp/engine_test.cpp), compiled here against the built library: host-only checks
on every machine, the forward on a GPU."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _build(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no C++ compiler")
    from oracle import oracle
    oracle.build()
    exe = tmp_path / "engine_test"
    libs = f"{ROOT / 'rustane_b200'}:{ROOT / 'oracle'}"
    cc = subprocess.run([gxx, "-std=c++17", "-O1", "-Wall", "-Wextra", "-Wpedantic", "-Wshadow", "-Werror",
                         f"-I{ROOT / 'include'}", str(ROOT / "tests" / "cpp" / "engine_test.cpp"),
                         f"-L{ROOT / 'rustane_b200'}", "-lcudabridge", f"-L{ROOT / 'oracle'}",
                         "-loracle", f"-Wl,-rpath,{libs}", "-pthread", "-o", str(exe)],
                        capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr[-3000:]
    return exe


def _run(exe, mode):
    r = subprocess.run([str(exe), mode], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert f"engine_test {mode}: ok" in r.stdout


def test_cpp_host_api_on_the_host(bridge_lib, tmp_path):
    _run(_build(tmp_path), "cpu")


@pytest.mark.gpu
def test_cpp_host_api_forward_on_gpu(bridge_lib, tmp_path):
    """forward_only_ws / forward / forward_losses / ForwardScheduler from C++ against the
    CPU oracle (loss within 1e-3 relative), host-array upload bit-equal to the device
    generator, workers' losses in request order."""
    _run(_build(tmp_path), "gpu")
