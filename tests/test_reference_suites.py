"""The reference's own test programs, compiled UNCHANGED against this build's drop-in headers and sources.

oracle/Makefile builds them from the reference tree (which only the build host has) into oracle/_ref/, mapping
the reference's include paths onto include/strata_kv/ through oracle/shim/.  Each program is the reference's
check-and-exit suite; passing it means the drop-in behaves as the reference's own tests require:
  conversation_cache_test   ConversationCache / ConversationBuffer / the prefix rules   (4,282 checks)
  conv_cache_test           the checkpoint-chain policy against the parked-conversation cache
  saved_conv_wire_test      the SR4H codec: layout, round trips, ~30 surgical refusals, slot sinks (483 checks)
  conversation_validation_test   (host-only build) the snapshot layer's refusals before any write, byte
                            estimates, layer carves and split stage sets (1,323 checks; CUDA is never initialised)
  handoff_arena_test        the hand-off table: on-disk layout, sizing, the claim/publish/release lifecycle,
                            dead and recycled owners, leases, refusals, cross-process readers, a >1 GiB slot and
                            an instance restart (268 checks; child processes, a tmpfs arena under /dev/shm)
The host suites run a second time as asan_* builds: this build's host sources compiled into the program with
AddressSanitizer and UndefinedBehaviorSanitizer, LeakSanitizer on at exit.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref")


@pytest.mark.parametrize("name,expect", [("ref_conversation_cache_test", "4282 checks passed"),
                                         ("ref_conv_cache_test", "PASS"),
                                         ("ref_saved_conv_wire_test", "483 checks passed"),
                                         ("ref_conversation_validation_test", "1323 host-only checks passed"),
                                         ("ref_handoff_arena_test", "268 checks, OK")])
def test_reference_suite_passes_against_the_drop_in(name, expect):
    path = os.path.join(BIN, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not built (the reference tree was not present at build time)")
    r = subprocess.run([path], capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert expect in r.stdout


@pytest.mark.parametrize("name,expect", [("asan_conversation_cache_test", "4282 checks passed"),
                                         ("asan_saved_conv_wire_test", "483 checks passed"),
                                         ("asan_conversation_validation_test", "1323 host-only checks passed"),
                                         ("asan_handoff_arena_test", "268 checks, OK")])
def test_reference_suite_passes_under_the_sanitizers(name, expect):
    path = os.path.join(BIN, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not built (the reference tree was not present at build time)")
    r = subprocess.run([path], capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES="",
                                ASAN_OPTIONS="protect_shadow_gap=0:detect_leaks=1:abort_on_error=0",
                                UBSAN_OPTIONS="print_stacktrace=1:halt_on_error=1"))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert expect in r.stdout
    assert "runtime error" not in r.stderr and "ERROR: AddressSanitizer" not in r.stderr
