"""The deadline the strip-sharded engine puts on its waits (hat-rs_b200/csrc/deadline.h),
checked on the CPU with fake probes: a peer that dies or stops calling must turn into an
error return after the deadline (or at once on the communicator's asynchronous error),
with the communicator aborted exactly once, never into a call that blocks forever."""
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_deadline_wait_outcomes(tmp_path):
    exe = tmp_path / "deadline_check"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(ROOT / "hat-rs_b200" / "csrc"),
                    str(ROOT / "tests" / "native" / "deadline_check.cpp"), "-o", str(exe), "-pthread"],
                   check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("ok ") == 5


def test_pass_rendezvous(tmp_path):
    """The host rendezvous that starts each strip-sharded pass (hat-rs_b200/csrc/rendezvous.h):
    a rank whose peer stops calling gets its error at the deadline with nothing enqueued, can
    repeat the call, and meets the peer again when it comes back; under races with short
    deadlines no rank ever proceeds before all have arrived."""
    exe = tmp_path / "rendezvous_check"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(ROOT / "hat-rs_b200" / "csrc"),
                    str(ROOT / "tests" / "native" / "rendezvous_check.cpp"), "-o", str(exe), "-pthread", "-lrt"],
                   check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("ok ") == 6
