"""The reference's own Catch2 attention test (ROCmKernels.Tests/AttentionTests.cpp), compiled
unchanged from its source against this library (oracle/_ref/attention_tests, see
oracle/Makefile), run on the GPU. Its CPU ReferenceAttention is the checker; its seven
sections call the library through the namespaced throwing wrappers."""
from __future__ import annotations

import subprocess

import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not oracle.REFERENCE_TESTS.exists(), reason="reference test binary not built (needs the reference tree)")
def test_reference_attention_tests_pass(cuda):
    result = subprocess.run([str(oracle.REFERENCE_TESTS), "-s"], capture_output=True, text=True, timeout=300)
    print(result.stdout)
    assert result.returncode == 0, result.stdout + result.stderr
    assert result.stdout.count("PASS:") == 7


@pytest.mark.skipif(not oracle.REFERENCE_GENERIC_TESTS.exists(),
                    reason="reference generic test binary not built (needs the reference tree)")
def test_reference_generic_tests_pass(cuda):
    """ROCmKernels.Tests/Generic/AttentionGenericTests.cpp, unchanged: head widths 16/32/64 x
    fp32/fp16, each leaf section two cases against its double-precision ComputeReference with
    its own max-abs tolerances (5e-4 fp32, 2e-3 fp16)."""
    result = subprocess.run([str(oracle.REFERENCE_GENERIC_TESTS), "-s"], capture_output=True, text=True, timeout=300)
    print(result.stdout)
    assert result.returncode == 0, result.stdout + result.stderr
    assert result.stdout.count("PASS:") == 6


@pytest.mark.skipif(not oracle.REFERENCE_POSITIONAL_TESTS.exists(),
                    reason="reference positional test binary not built (needs the reference tree)")
def test_reference_positional_tests_pass(cuda):
    """ROCmKernels.Tests/PositionalTests.cpp, unchanged: the rotary forward and backward cases
    against its ReferenceRotary with its 1e-6 max-abs bar."""
    result = subprocess.run([str(oracle.REFERENCE_POSITIONAL_TESTS), "-s"], capture_output=True, text=True, timeout=300)
    print(result.stdout)
    assert result.returncode == 0, result.stdout + result.stderr
    assert result.stdout.count("PASS:") == 2
