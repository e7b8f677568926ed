"""The GPU suite again on the bounds-checking debug build.

lib/libwgx_bounds.so is compiled with -DWGX_BOUNDS: every global store,
residual load, operand copy and staging read of the tensor-core convolution
(umma_conv_kernel, its input packers) and of the sliding-window depthwise
kernel checks its address range against the extent of the buffer it
targets, skips an access that falls outside and raises the kErrBounds bit of
the device error word, which the next wgx_sync reports as WGX_ERR_DEVICE.
Running every GPU parity, model, noalloc and failure test on that library
in a child process shows that none of their launches ever reaches outside a
buffer, without a memory checker on the device.
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "wgpu-executorch_b200", "lib", "libwgx_bounds.so")


@pytest.mark.gpu
def test_gpu_suite_on_bounds_checking_build():
    assert os.path.exists(LIB), "bounds build missing: make -C wgpu-executorch_b200 bounds"
    env = dict(os.environ, WGX_LIBRARY="bounds")
    # the child must really run on the bounds library
    probe = subprocess.run(
        [sys.executable, "-c",
         "import sys; sys.path.insert(0, 'wgpu-executorch_b200'); from wgx import _lib; "
         "print(_lib.LIB_PATH, _lib.build_flags())"],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert probe.returncode == 0, probe.stderr
    path, flags = probe.stdout.split()
    assert path == LIB and int(flags) == 1
    r = subprocess.run(
        [sys.executable, "-m", "pytest", "tests", "-m", "gpu", "-x", "-q", "-p", "no:cacheprovider",
         "--ignore", os.path.join("tests", "test_gpu_bounds.py")],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=1800)
    tail = "\n".join((r.stdout + r.stderr).splitlines()[-30:])
    assert r.returncode == 0, tail
    assert " passed" in tail and "failed" not in tail, tail
