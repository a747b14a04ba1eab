"""Comparison helpers shared by the parity tests (the reference grader's rule)."""

import numpy as np

from oracle.ops import bf16_to_f32

# Per-op tolerances of the reference grader (furiosa-opt-gemma4-12B/src/bin/test_kernels.rs:447-465).
RTOL = 1e-2
ATOL = {"sliding_project_qkv": 0.04, "sliding_attention_output": 0.05, "decoder_feedforward": 0.01}


def within(expected_bits, actual_bits, atol, rtol=RTOL):
    """|want - got| <= atol + rtol * |want| for every element, and no non-finite output
    (test_kernels.rs:626-671). Returns (ok, max_abs_diff, fraction_bit_exact)."""
    want = bf16_to_f32(np.asarray(expected_bits).reshape(-1))
    got = bf16_to_f32(np.asarray(actual_bits).reshape(-1))
    assert want.shape == got.shape, (want.shape, got.shape)
    finite = np.isfinite(got).all()
    diff = np.abs(want - got)
    ok = bool(finite and (diff <= atol + rtol * np.abs(want)).all())
    exact = float(np.mean(np.asarray(expected_bits).reshape(-1) == np.asarray(actual_bits).reshape(-1)))
    return ok, float(diff.max()) if diff.size else 0.0, exact
