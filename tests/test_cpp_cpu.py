"""Host-only C++ test programs (tests/cpp/*_cpu_test.cpp), built against libstrata_kv.so and run here.

handoff_device_cpu_test: the 256-byte device descriptor a hand-off slot carries on one node - round trip, every
refusal, and its trip through a real HandoffArena slot (claim, write, publish, read, release).
wire_fuzz_cpu_test: the SR4H decoders (full and shape) against damaged copies of the reference's own payloads,
compiled from the sources with AddressSanitizer and UndefinedBehaviorSanitizer.
c_abi_cpu_test: include/strata_kv.h compiled as pedantic C99 with warnings as errors, and the entry points that
need no GPU called from C.
arena_fuzz_cpu_test: the hand-off arena reader against damaged arena files (headers, sizes), under the sanitizers.
arena_threads_cpu_test: one arena shared by four threads (claim, publish, read, release), under ThreadSanitizer.
"""
import os
import subprocess
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp")
BIN = os.path.join(SRC, "bin")
PKG = os.path.join(ROOT, "strata-concurrent_b200")
CUDA = "/usr/local/cuda"


def build(name: str) -> str:
    os.makedirs(BIN, exist_ok=True)
    src = os.path.join(SRC, name + ".cpp")
    out = os.path.join(BIN, name)
    deps = [src, os.path.join(PKG, "libstrata_kv.so")]
    if not os.path.exists(out) or any(os.path.getmtime(d) > os.path.getmtime(out) for d in deps):
        subprocess.run(["g++", "-std=c++20", "-O2", "-I", os.path.join(ROOT, "include"), "-I", f"{CUDA}/include",
                        "-o", out, src, "-L", PKG, "-lstrata_kv", f"-Wl,-rpath,{PKG}", "-L", f"{CUDA}/lib64",
                        "-lcudart", f"-Wl,-rpath,{CUDA}/lib64"], check=True)
    return out


def test_device_descriptor_round_trip_refusals_and_slot():
    exe = build("handoff_device_cpu_test")
    with tempfile.TemporaryDirectory() as d:
        r = subprocess.run([exe, d], capture_output=True, text=True, timeout=300,
                           env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "checks passed" in r.stdout


def test_wire_decoders_refuse_damaged_payloads_without_a_bad_access():
    os.makedirs(BIN, exist_ok=True)
    out = os.path.join(BIN, "wire_fuzz_cpu_test")
    host = os.path.join(PKG, "csrc", "host")
    srcs = [os.path.join(SRC, "wire_fuzz_cpu_test.cpp"), os.path.join(host, "conversation_wire.cpp"),
            os.path.join(host, "pinned.cpp")]
    deps = srcs + [os.path.join(host, "wire_detail.hpp")] + [
        os.path.join(ROOT, "include", "strata_kv", h) for h in ("conversation_wire.hpp", "conversation_cache.hpp",
                                                                 "conversation_buffer.hpp")]
    if not os.path.exists(out) or any(os.path.getmtime(d) > os.path.getmtime(out) for d in deps):
        subprocess.run(["g++", "-std=c++20", "-O1", "-g", "-fsanitize=address,undefined",
                        "-fno-sanitize-recover=undefined", "-fno-omit-frame-pointer", "-I", os.path.join(ROOT, "include"),
                        "-I", host, "-I", f"{CUDA}/include", "-o", out, *srcs, "-L", f"{CUDA}/lib64", "-lcudart",
                        f"-Wl,-rpath,{CUDA}/lib64"], check=True)
    golden = os.path.join(ROOT, "tests", "golden")
    payloads = [os.path.join(golden, f"ref_payload_T{t}.bin") for t in (1, 5, 257)]
    r = subprocess.run([out, "3000", *payloads], capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES="", ASAN_OPTIONS="protect_shadow_gap=0:detect_leaks=0"))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert ", OK" in r.stdout


def test_the_c_header_is_c_and_the_host_entry_points_work_from_c():
    os.makedirs(BIN, exist_ok=True)
    src = os.path.join(SRC, "c_abi_cpu_test.c")
    out = os.path.join(BIN, "c_abi_cpu_test")
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", os.path.join(ROOT, "include"),
                    "-o", out, src, "-L", PKG, "-lstrata_kv", f"-Wl,-rpath,{PKG}", "-L", f"{CUDA}/lib64", "-lcudart",
                    f"-Wl,-rpath,{CUDA}/lib64"], check=True)
    r = subprocess.run([out], capture_output=True, text=True, timeout=120, env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert ", OK" in r.stdout


def test_every_cxx_header_stands_alone_and_compiles_clean():
    """Each include/strata_kv/*.hpp compiles as the only include of a translation unit (twice, for the guard) with
    -Wall -Wextra -Wpedantic -Wshadow -Werror: what a maintainer's target includes needs nothing else first."""
    hdr_dir = os.path.join(ROOT, "include", "strata_kv")
    names = sorted(n for n in os.listdir(hdr_dir) if n.endswith(".hpp"))
    assert names
    with tempfile.TemporaryDirectory() as d:
        for n in names:
            tu = os.path.join(d, "tu.cpp")
            with open(tu, "w") as f:
                f.write(f'#include "strata_kv/{n}"\n#include "strata_kv/{n}"\n')
            r = subprocess.run(["g++", "-std=c++20", "-Wall", "-Wextra", "-Wpedantic", "-Wshadow", "-Werror",
                                "-fsyntax-only", "-I", os.path.join(ROOT, "include"), "-I", f"{CUDA}/include", tu],
                               capture_output=True, text=True, timeout=120)
            assert r.returncode == 0, n + ": " + r.stderr[-2000:]


def test_arena_reader_refuses_damaged_arena_files_without_a_bad_access():
    os.makedirs(BIN, exist_ok=True)
    out = os.path.join(BIN, "arena_fuzz_cpu_test")
    host = os.path.join(PKG, "csrc", "host")
    srcs = [os.path.join(SRC, "arena_fuzz_cpu_test.cpp"), os.path.join(host, "handoff.cpp"),
            os.path.join(host, "conversation_wire.cpp"), os.path.join(host, "pinned.cpp")]
    deps = srcs + [os.path.join(ROOT, "include", "strata_kv", "handoff.hpp")]
    if not os.path.exists(out) or any(os.path.getmtime(d) > os.path.getmtime(out) for d in deps):
        subprocess.run(["g++", "-std=c++20", "-O1", "-g", "-fsanitize=address,undefined",
                        "-fno-sanitize-recover=undefined", "-fno-omit-frame-pointer", "-I", os.path.join(ROOT, "include"),
                        "-I", host, "-I", f"{CUDA}/include", "-o", out, *srcs, "-L", f"{CUDA}/lib64", "-lcudart",
                        f"-Wl,-rpath,{CUDA}/lib64", "-pthread"], check=True)
    with tempfile.TemporaryDirectory() as d:
        r = subprocess.run([out, d, "2000"], capture_output=True, text=True, timeout=600,
                           env=dict(os.environ, CUDA_VISIBLE_DEVICES="",
                                    ASAN_OPTIONS="protect_shadow_gap=0:detect_leaks=1"))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert ", OK" in r.stdout


def test_one_arena_shared_by_threads_has_no_data_race():
    os.makedirs(BIN, exist_ok=True)
    out = os.path.join(BIN, "arena_threads_cpu_test")
    host = os.path.join(PKG, "csrc", "host")
    srcs = [os.path.join(SRC, "arena_threads_cpu_test.cpp"), os.path.join(host, "handoff.cpp"),
            os.path.join(host, "conversation_wire.cpp"), os.path.join(host, "pinned.cpp")]
    deps = srcs + [os.path.join(ROOT, "include", "strata_kv", "handoff.hpp")]
    if not os.path.exists(out) or any(os.path.getmtime(d) > os.path.getmtime(out) for d in deps):
        subprocess.run(["g++", "-std=c++20", "-O1", "-g", "-fsanitize=thread", "-Wno-tsan", "-I",
                        os.path.join(ROOT, "include"), "-I", host, "-I", f"{CUDA}/include", "-o", out, *srcs,
                        "-L", f"{CUDA}/lib64", "-lcudart", f"-Wl,-rpath,{CUDA}/lib64", "-pthread"], check=True)
    with tempfile.TemporaryDirectory() as d:
        r = subprocess.run([out, d], capture_output=True, text=True, timeout=600,
                           env=dict(os.environ, CUDA_VISIBLE_DEVICES="", TSAN_OPTIONS="halt_on_error=1"))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert ", OK" in r.stdout and "WARNING: ThreadSanitizer" not in r.stderr


def test_the_documented_integration_calls_compile():
    """tests/cpp/integration_snippets_cpu_test.cpp holds the calls that bind this library into the reference
    engine, written over the engine's types: they must keep compiling against the headers."""
    r = subprocess.run(["g++", "-std=c++20", "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-I",
                        os.path.join(ROOT, "include"), "-I", f"{CUDA}/include",
                        os.path.join(SRC, "integration_snippets_cpu_test.cpp")], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr[-3000:]
