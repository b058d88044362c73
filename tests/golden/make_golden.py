"""Generates the golden vectors in tests/golden/ from the reference's own code.

Run where the reference tree is available (it is not on the GPU box):

    make -C oracle oracle ref && python tests/golden/make_golden.py

For every case, the inputs come from the reference's ``RandomValues`` (TestSupport.hpp:11-21)
and the expected outputs from the reference's ``ReferenceAttention``
(ROCmKernels.Tests/AttentionTests.cpp:28-125). Both run from the reference's source, compiled
in place into oracle/_ref/libref_attention.so. The seven cases named ``reference_*`` are the
sections of AttentionTests.cpp:272-286 (seeds 101-104, U(-1,1), mask[3] = 0). The ``extra_*``
cases add what those sections do not cover: Q != K with a radius, a fully masked sequence, and
a 64-wide masked radius case.

The ``rotary_*`` cases pin the rotary oracle: inputs from ``RandomValues`` (q, k in [-2, 2),
cos, sin in [-1, 1)) and outputs from the reference's ``ReferenceRotary``
(ROCmKernels.Tests/PositionalTests.cpp:18-50, compiled in place into
oracle/_ref/libref_positional.so); ``rotary_reference_*`` are that file's two test cases (:53-141).

``normal_pin.npz`` holds the first values of std::normal_distribution<float>(0, 1) over
std::mt19937(seed). They come from a small C++ program compiled with g++, and pin the
oracle's restatement of the libstdc++ normal distribution used for the benchmark inputs.
"""
from __future__ import annotations

import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import oracle  # noqa: E402

# name: (head_width, batch, heads, queries, keys, radius, upstream_zero, masked_batches)
CASES = {
    "reference_simple_d32": (32, 2, 2, 4, 6, -1, False, ()),      # AttentionTests.cpp:273
    "reference_tiled_d32": (32, 1, 1, 40, 40, -1, False, ()),     # :275
    "reference_flash_d32": (32, 1, 2, 40, 40, -1, True, ()),      # :277
    "reference_flash_banded_d32": (32, 1, 2, 64, 64, 5, True, ()),  # :279
    "reference_flash_variant8_d32": (32, 1, 1, 40, 40, -1, True, ()),  # :281
    "reference_flash_variant1_d32": (32, 1, 1, 40, 40, -1, True, ()),  # :283
    "reference_simple_d64": (64, 1, 2, 4, 6, -1, False, ()),      # :285
    "extra_radius_ragged_d32": (32, 2, 3, 50, 70, 7, False, ()),
    "extra_masked_sequence_d32": (32, 2, 2, 33, 17, -1, False, (1,)),
    "extra_radius_masked_d64": (64, 2, 2, 37, 29, 3, False, (1,)),
}

# name: (batch, heads, length, backward, seeds of q, k, cos, sin)
ROTARY_CASES = {
    "rotary_reference_forward": (2, 3, 4, False, (21, 22, 23, 24)),   # PositionalTests.cpp:53-96
    "rotary_reference_backward": (1, 2, 3, True, (31, 32, 33, 34)),   # :98-141
    "rotary_extra_forward": (3, 5, 37, False, (41, 42, 43, 44)),
    "rotary_extra_backward": (2, 4, 29, True, (51, 52, 53, 54)),
}

NORMAL_SOURCE = r"""
#include <cstdio>
#include <cstdlib>
#include <random>
int main(int argc, char **argv) {
    std::mt19937 engine(std::strtoul(argv[1], nullptr, 10));
    std::normal_distribution<float> normal(0.0f, 1.0f);
    const long count = std::strtol(argv[2], nullptr, 10);
    for (long i = 0; i < count; ++i) { float v = normal(engine); std::fwrite(&v, 4, 1, stdout); }
}
"""


def make_case(head_width, batch, heads, queries, keys, radius, upstream_zero, masked_batches):
    qn, kn = batch * heads * queries * head_width, batch * heads * keys * head_width
    q = oracle.reference_random_values(qn, 101).reshape(batch, heads, queries, head_width)
    k = oracle.reference_random_values(kn, 102).reshape(batch, heads, keys, head_width)
    v = oracle.reference_random_values(kn, 103).reshape(batch, heads, keys, head_width)
    if upstream_zero:
        upstream = np.zeros_like(q)
    else:
        upstream = oracle.reference_random_values(qn, 104).reshape(q.shape)
    mask = np.ones((batch, keys), np.uint8)
    mask.flat[3] = 0
    for b in masked_batches:
        mask[b, :] = 0
    expected = oracle.reference_attention(q, k, v, mask, upstream, radius)
    return dict(q=q, k=k, v=v, upstream=upstream, mask=mask, radius=np.int32(radius), **expected)


def make_rotary_case(batch, heads, length, backward, seeds):
    elements, table = batch * heads * length * 32, batch * length * 32
    q = oracle.reference_random_values(elements, seeds[0], -2.0, 2.0).reshape(batch, length, heads, 32)
    k = oracle.reference_random_values(elements, seeds[1], -2.0, 2.0).reshape(batch, length, heads, 32)
    cos = oracle.reference_random_values(table, seeds[2], -1.0, 1.0).reshape(batch, length, 32)
    sin = oracle.reference_random_values(table, seeds[3], -1.0, 1.0).reshape(batch, length, 32)
    return dict(q=q, k=k, cos=cos, sin=sin, backward=np.int32(backward), seeds=np.int32(seeds),
                out_q=oracle.reference_rotary(q, cos, sin, backward), out_k=oracle.reference_rotary(k, cos, sin, backward))


def normal_pin(seed: int, count: int) -> np.ndarray:
    with tempfile.TemporaryDirectory() as tmp:
        source = Path(tmp) / "normal.cpp"
        source.write_text(NORMAL_SOURCE)
        binary = Path(tmp) / "normal"
        subprocess.run(["g++", "-O2", "-o", str(binary), str(source)], check=True)
        raw = subprocess.run([str(binary), str(seed), str(count)], check=True, capture_output=True).stdout
    return np.frombuffer(raw, dtype=np.float32).copy()


def main() -> None:
    if not oracle.reference_available():
        raise SystemExit("oracle/_ref/libref_attention.so is missing: run `make -C oracle ref` where the reference exists")
    for name, spec in CASES.items():
        np.savez_compressed(HERE / f"{name}.npz", **make_case(*spec))
        print("wrote", name)
    np.savez_compressed(HERE / "normal_pin.npz", seed101=normal_pin(101, 4096), seed105=normal_pin(105, 4096))
    print("wrote normal_pin")
    if not oracle.reference_positional_available():
        raise SystemExit("oracle/_ref/libref_positional.so is missing: run `make -C oracle ref` where the reference exists")
    for name, spec in ROTARY_CASES.items():
        np.savez_compressed(HERE / f"{name}.npz", **make_rotary_case(*spec))
        print("wrote", name)


if __name__ == "__main__":
    main()
