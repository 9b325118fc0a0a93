"""Generate the golden fixtures for the MLA decode oracle.

Runs the reference's OWN FP32 CPU kernel (``run_mla_decode_cpu``, lechebs/ada-mla
csrc/mla_decode_naive_fp32_cpu.cpp:5-61, compiled unchanged from the reference
sources into ``oracle/_ref/`` by ``make -C oracle ref``) on small seeded inputs
and stores inputs and outputs in ``tests/golden/mla_ref_golden.npz``.

The reference has no golden vectors or known-answer tests of its own, so these
fixtures are the pin for the oracle restatement (``oracle/mla_oracle.c``) and,
through it, for the CUDA kernels.  Run from the repository root:

    make -C oracle ref && python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mla_ref_golden.npz")

# (name, num_heads, seq_length, kind)
#   "raw":    fp32 N(0,1) Q and C, the reference's own calling convention
#             (internal 1/sqrt(576) scale, all 576 output columns).
#   "folded": BASELINE-style inputs: C ~ N(0,1) and Q ~ N(0,1)/sqrt(192), both
#             rounded to fp16, with Q pre-multiplied by sqrt(576) so the kernel's
#             internal division leaves softmax(Q* C^T).
CASES = [
    ("raw_h4_n17", 4, 17, "raw"),
    ("raw_h16_n33", 16, 33, "raw"),
    ("raw_h8_n1", 8, 1, "raw"),
    ("raw_h2_n130", 2, 130, "raw"),
    ("folded_h128_n20", 128, 20, "folded"),
    ("folded_h16_n100", 16, 100, "folded"),
]


def main() -> None:
    if not oracle.have_ref():
        raise SystemExit("oracle/_ref/libref_mla_cpu.so missing: run `make -C oracle ref` first")
    arrays: dict[str, np.ndarray] = {}
    for i, (name, nh, n, kind) in enumerate(CASES):
        rng = np.random.default_rng(1000 + i)
        q = rng.standard_normal((nh, 576), dtype=np.float32)
        c = rng.standard_normal((n, 576), dtype=np.float32)
        if kind == "folded":
            q = (q / np.sqrt(192.0)).astype(np.float16)
            c = c.astype(np.float16)
            q_in = (q.astype(np.float32) * np.float32(24.0)).astype(np.float32)
            out = oracle.run_mla_decode_cpu(q_in, c.astype(np.float32), impl="reference")
        else:
            out = oracle.run_mla_decode_cpu(q, c, impl="reference")
        arrays[f"{name}__q"] = q
        arrays[f"{name}__c"] = c
        arrays[f"{name}__out"] = out
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(CASES)} cases)")


if __name__ == "__main__":
    main()
