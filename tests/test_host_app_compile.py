"""The named-global host ABI (include/sched/sched_rt.h) builds into a CUDA
host application for sm_100a (examples/host_app_sched_rt.cu), and without a
usable GPU its initialisation fails with a message and a non-zero exit
instead of crashing."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("nvcc") is None and not os.path.exists("/usr/local/cuda/bin/nvcc"),
                    reason="needs nvcc")
def test_host_app_builds_and_fails_cleanly_without_a_gpu(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / "host_app"
    r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17",
                        "-I" + os.path.join(ROOT, "include"), "-o", str(exe),
                        os.path.join(ROOT, "examples", "host_app_sched_rt.cu")],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the GPU run belongs to the gpu tests")
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60,
                         env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert run.returncode == 1 and "[sched_rt]" in run.stderr
