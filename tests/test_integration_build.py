"""The drop-in boundary, built: integration/executor.patch applied to the reference's
own sources plus integration/{include,src} (CudaExecutable, device tensors), compiled by
integration/Makefile into a reference library whose Executor has ExecutionMode::
CompiledCUDA and links libtt_cuda.so.  These host checks need no GPU: the patch applies,
the library and the patched Python module build and load, and on a machine without a
GPU the CUDA mode fails the way the reference reports runtime errors
(RuntimeExecutionError) instead of falling back to a CPU path.  The GPU runs are in
tests/test_gpu_integration.py."""

import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
INTEG = os.path.join(ROOT, "integration")
LIB = os.path.join(INTEG, "_build", "libttref_cuda.so")
PKG = os.path.join(INTEG, "_build", "pkg")
REF = "/root/reference"


def _have_gpu():
    import torch

    return torch.cuda.is_available()


@pytest.fixture(scope="module")
def built():
    """Builds the integration library (and Python module) where the reference sources
    exist; elsewhere uses the files built with the snapshot, or skips."""
    if os.path.isdir(os.path.join(REF, "src")):
        subprocess.run(["make", "-s", "-C", INTEG, "-j8", "all", "py"], check=True)
    if not os.path.exists(LIB):
        pytest.skip("integration library not built (no reference sources here)")
    return LIB


def test_patch_applies_to_the_reference_sources(tmp_path):
    if not os.path.isdir(os.path.join(REF, "src")):
        pytest.skip("reference sources absent")
    for d in ("include", "src", "bindings", "python"):
        subprocess.run(["cp", "-r", os.path.join(REF, d), str(tmp_path)], check=True)
    r = subprocess.run(["patch", "--dry-run", "-p1", "-d", str(tmp_path), "-i", os.path.join(INTEG, "executor.patch")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    for f in ("include/tinytensor/runtime/executor.hpp", "src/runtime/executor.cpp",
              "bindings/python_bindings.cpp", "python/tinytensor/compiler.py"):
        assert f"checking file {f}" in r.stdout


def test_library_links_the_cuda_backend(built):
    out = subprocess.run(["ldd", built], capture_output=True, text=True).stdout
    line = [ln for ln in out.splitlines() if "libtt_cuda.so" in ln]
    assert line and "not found" not in line[0], out
    assert os.path.samefile(line[0].split("=>")[1].split("(")[0].strip(),
                            os.path.join(ROOT, "tinytensor_b200", "lib", "libtt_cuda.so"))
    lib = ctypes.CDLL(built)
    assert lib.ttref_has_cuda() == 1


def test_cuda_mode_without_a_gpu_raises_runtime_execution_error(built):
    if _have_gpu():
        pytest.skip("a GPU is present")
    sys.path.insert(0, ROOT)
    from oracle import oracle as O

    import tinytensor_b200 as tt

    R = O.Reference(built)
    g = tt.Graph()
    a, b = g.input([4, 8]), g.input([4, 8])
    y = tt.relu(a + b)
    with pytest.raises(RuntimeError, match="RuntimeExecutionError: no device"):
        R.run(g, {a: np.ones((4, 8), np.float32), b: np.ones((4, 8), np.float32)}, mode="cuda", outputs=[y])
    # the other modes of the same (patched) library still work
    out = R.run(g, {a: np.ones((4, 8), np.float32), b: np.ones((4, 8), np.float32)}, mode="interpreted", outputs=[y])
    assert np.array_equal(out[0], np.full((4, 8), 2.0, np.float32))


def test_python_module_has_the_cuda_mode(built):
    if not os.path.isdir(os.path.join(PKG, "tinytensor")):
        pytest.skip("patched Python package not built")
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "import tinytensor as tt\n"
        "from tinytensor._tinytensor import ExecutionMode, cuda_to_device, cuda_is_device\n"
        "assert hasattr(ExecutionMode, 'CompiledCUDA')\n"
        "g = tt.Graph(); a = g.input([2, 3]); y = g.relu(a)\n"
        "try:\n"
        "    tt.compile(g, outputs=[y], mode='cuda')\n"
        "    print('compiled')\n"
        "except Exception as e:\n"
        "    print(type(e).__name__, e)\n" % PKG
    )
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    if not _have_gpu():
        assert "no device" in r.stdout, r.stdout
