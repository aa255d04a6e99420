"""Host-only logic of the library on CPU, with stubbed CUDA and NCCL calls
(tests/native/host_logic_test.cpp over csrc/hb_host.h): the static scratch's
address cache follows the device's context (a reset context is looked up
again, never reused), and the ring's host wait ends on completion, on a
communicator error, on a failed stream query, or at its deadline."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_host_logic(tmp_path):
    exe = tmp_path / "host_logic_test"
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-pthread",
                    "-I", os.path.join(ROOT, "herbert-jit-bf16_b200", "csrc"),
                    "-o", str(exe), os.path.join(ROOT, "tests", "native", "host_logic_test.cpp")],
                   check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
