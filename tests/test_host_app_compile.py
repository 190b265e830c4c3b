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


@pytest.mark.gpu
def test_host_app_runs_on_the_gpu(tmp_path):
    """The host application on a B200: sched_rt_init arms the named device
    globals, a reversed task order is honoured (every task computes its own
    slot), the timer fills exactly one row per task on the armed launch,
    sched_rt_disarm returns the kernel to its stock path, and the JSON
    publication names the device slots."""
    import json
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / "host_app"
    r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17",
                        "-I" + os.path.join(ROOT, "include"), "-o", str(exe),
                        os.path.join(ROOT, "examples", "host_app_sched_rt.cu")],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout[-2000:] + run.stderr[-2000:]
    lines = run.stdout.strip().splitlines()
    assert lines[-1] == "OK"
    pub = json.loads("\n".join(lines[:-1]))
    for key in ("pid", "max_tasks", "order_dev", "ctrl_dev", "timer_host_va", "timer_bytes", "queue_dev"):
        assert key in pub, pub
    assert pub["order_dev"] and pub["ctrl_dev"] and pub["timer_bytes"] == 8 * pub["max_tasks"]
