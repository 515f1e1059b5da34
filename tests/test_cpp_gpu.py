"""The C++ drop-in API on a real device (tests/cpp/*.cpp, reference-style check-and-exit programs).

snapshot_gpu_test parks config 1 (full geometry, 4,096 tokens, seed 1) from a pool at seed-random slots with
conversation_snapshot_save, and the SR4H payload of the parked image must hash to the FNV-1a the reference's own
save + encode produced from its identity pool (tests/golden/golden.json).  It then mounts the image into a
differently permuted pool and reads every byte back; see the program's header for the full list.

kv_stream_gpu_test checks the block movers of streamed and ring layers (reset, the CLOCK resolve against the
oracle's sequential restatement, ring table / restore, stage from host).

The reference's own GPU test program, conversation_snapshot_test (built unchanged against this build by
oracle/Makefile), parks and mounts every KV format in resident, streamed and ring layers, whole and layer-split.
"""
import json
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp")
BIN = os.path.join(SRC, "bin")
PKG = os.path.join(ROOT, "strata-concurrent_b200")
ORACLE = os.path.join(ROOT, "oracle")
CUDA = "/usr/local/cuda"


HOST_INTERNALS = os.path.join(PKG, "csrc", "host")   # the library's internal headers (the transfer fault seam)


def build(name: str) -> str:
    os.makedirs(BIN, exist_ok=True)
    src = os.path.join(SRC, name + ".cpp")
    out = os.path.join(BIN, name)
    deps = [src, os.path.join(SRC, "session_fixture.hpp"), os.path.join(PKG, "libstrata_kv.so"),
            os.path.join(ORACLE, "liboracle.so")]
    if not os.path.exists(out) or any(os.path.getmtime(d) > os.path.getmtime(out) for d in deps):
        subprocess.run(["g++", "-std=c++20", "-O2", "-I", os.path.join(ROOT, "include"), "-I", ORACLE,
                        "-I", HOST_INTERNALS,
                        "-I", f"{CUDA}/include", "-o", out, src, "-L", PKG, "-lstrata_kv", f"-Wl,-rpath,{PKG}",
                        "-L", ORACLE, "-loracle", f"-Wl,-rpath,{ORACLE}", "-L", f"{CUDA}/lib64", "-lcudart",
                        f"-Wl,-rpath,{CUDA}/lib64"], check=True)
    return out


def test_snapshot_park_mount_matches_reference_payload(torch_cuda):
    golden = json.load(open(os.path.join(ROOT, "tests", "golden", "golden.json")))["config1"]
    exe = build("snapshot_gpu_test")
    r = subprocess.run([exe, str(golden["bytes"]), str(golden["payload_hash"])], capture_output=True, text=True,
                       timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "checks passed" in r.stdout


def test_kv_stream_block_movers_match_the_oracle(torch_cuda):
    exe = build("kv_stream_gpu_test")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "checks passed" in r.stdout


def test_reference_gpu_snapshot_suite_passes_against_the_drop_in(torch_cuda):
    exe = os.path.join(ORACLE, "_ref", "ref_conversation_snapshot_test")
    if not os.path.exists(exe):
        pytest.skip("ref_conversation_snapshot_test not built (the reference tree was not present at build time)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "conversation_snapshot_test:" in r.stdout and "checks passed" in r.stdout


@pytest.mark.parametrize("tokens", [4096, 32768])
def test_split_role_handoff_through_a_device_descriptor(torch_cuda, tokens):
    """Two processes, two GPUs: the prefill instance publishes a device descriptor in a hand-off slot, the decode
    instance mounts straight from the prefill GPU's HBM (see the program's header)."""
    if torch_cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import tempfile
    exe = build("handoff_device_gpu_test")
    with tempfile.TemporaryDirectory() as d:
        r = subprocess.run([exe, d, str(tokens)], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "both instances passed" in r.stdout


def test_device_mount_agrees_with_host_mount_for_every_format_and_mode(torch_cuda):
    exe = build("device_mount_formats_gpu_test")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "checks passed" in r.stdout


def test_serve_slot_hand_overs_through_the_reference_serve_swap(torch_cuda):
    """Row a14, the callers: the reference's serve_swap::run drives park / validate / mount hooks written the way
    src/program/generate.cpp:4185-4266 and 5913-5940 write them, against this build, over three serve slots
    (tests/cpp/serve_swap_gpu_test.cpp; built by oracle/Makefile because it needs the reference's header)."""
    exe = os.path.join(ORACLE, "_ref", "serve_swap_gpu_test")
    if not os.path.exists(exe):
        pytest.skip("serve_swap_gpu_test not built (the reference tree was not present at build time)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "serve_swap_gpu_test:" in r.stdout and "checks passed" in r.stdout


def test_transfer_failures_injected_on_the_host(torch_cuda):
    """Every host-side step of a park and of a mount (device and stream synchronisations, host copies, copy-kernel
    launches) failed one at a time through the library's fault seam: the reference's transfer-failure cases
    (src/core/conversation_validation_test.cpp:171-195, 475-500) against this build's batches (see the program's
    header).  No GPU fault is involved."""
    exe = build("transfer_faults_gpu_test")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "transfer_faults_gpu_test:" in r.stdout and "checks passed" in r.stdout
