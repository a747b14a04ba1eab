"""CPU: pin the oracle to the reference's own golden vectors (no GPU needed).

- every synthesized input reproduces the reference fixture's checksum (byte-exact PRNG)
- the oracle's outputs match the reference oracle's outputs within the grader tolerance
- the constructed FFN-stress case reproduces its committed expectation bit for bit
- the QKV cancellation cases reproduce the reference's boundary-suite expectations
- the attention restatement agrees with gemma4.py's SDPA call and with a float64 softmax
"""

import numpy as np
import pytest

from oracle import ops, prng, synth
from helpers import ATOL, within

RUNS = range(9)


@pytest.mark.parametrize("run", RUNS)
def test_prng_checksums_match_reference(run, golden_runs):
    for test, build in (("sliding_project_qkv", synth.sliding_project_qkv),
                        ("sliding_attention_output", synth.sliding_attention_output),
                        ("decoder_feedforward", synth.decoder_feedforward)):
        d = build(run)
        for name, value in d["checks"].items():
            want = int(golden_runs[f"run{run}.{test}.check.{name}"][0]) & 0xFFFFFFFF
            assert value == want, f"run{run}.{test}.{name}: {value:#010x} != {want:#010x}"


def test_prng_c_and_numpy_agree(monkeypatch):
    """The C restatement (oracle/c/g4oracle.c) and the numpy definition produce the same bytes."""
    if prng._lib() is None:
        pytest.skip("oracle/_build/libg4oracle.so not built")
    n = 1 << 17
    c_f4, c_f8 = prng.f4_nibbles("t.f4", n), prng.f8_banded("t.f8", n, 8, 10, False)
    c_ck = prng.checksum(np.arange(1 << 21, dtype=np.uint32).view(np.uint8))
    monkeypatch.setenv("G4_ORACLE_NUMPY_ONLY", "1")
    monkeypatch.setattr(prng, "_LIB", None)
    assert np.array_equal(c_f4, prng.f4_nibbles("t.f4", n))
    assert np.array_equal(c_f8, prng.f8_banded("t.f8", n, 8, 10, False))
    assert c_ck == prng.checksum(np.arange(1 << 21, dtype=np.uint32).view(np.uint8))


def qkv_oracle(d):
    return ops.sliding_project_qkv(d["x"], d["q_weight"], d["k_weight"], d["v_weight"], d["q_weight_scale"],
                                   d["k_weight_scale"], d["v_weight_scale"], d["input_rms_weight"],
                                   d["q_rms_weight"], d["k_rms_weight"], d["cos_row"], d["sin_row"])


def ffn_oracle(d):
    return ops.decoder_feedforward(d["residual"], d["pre_ff_rms_weight"], d["up_weight_packed"],
                                   d["gate_weight_packed"], d["down_weight_packed"], d["up_weight_scale"],
                                   d["gate_weight_scale"], d["down_weight_scale"], d["up_global_scale"][0],
                                   d["gate_global_scale"][0], d["down_global_scale"][0], d["post_ff_rms_weight"],
                                   d["layer_scalar"])


@pytest.mark.parametrize("run", RUNS)
def test_oracle_qkv_matches_reference(run, golden_runs):
    q, k, v = qkv_oracle(synth.sliding_project_qkv(run))
    for label, got in (("q", q), ("k", k), ("v", v)):
        ok, maxd, exact = within(golden_runs[f"run{run}.sliding_project_qkv.expected.{label}"], got,
                                 ATOL["sliding_project_qkv"])
        assert ok and exact > 0.99, (label, maxd, exact)


@pytest.mark.parametrize("run", RUNS)
def test_oracle_o_matches_reference(run, golden_runs):
    d = synth.sliding_attention_output(run)
    got = ops.sliding_attention_output(d["x"], d["post_attn_rms_weight"], d["o_weight"], d["o_weight_scale"],
                                       d["residual"])
    ok, maxd, exact = within(golden_runs[f"run{run}.sliding_attention_output.expected"], got,
                             ATOL["sliding_attention_output"])
    assert ok and exact > 0.99, (maxd, exact)


@pytest.mark.parametrize("run", [0, 1, 2])
def test_oracle_ffn_matches_reference(run, golden_runs):
    got = ffn_oracle(synth.decoder_feedforward(run))
    ok, maxd, exact = within(golden_runs[f"run{run}.decoder_feedforward.expected"], got, ATOL["decoder_feedforward"])
    assert ok and exact > 0.95, (maxd, exact)


def test_oracle_ffn_stress_exact(golden_stress):
    d = synth.ffn_stress()
    got = ffn_oracle(d)
    assert np.array_equal(golden_stress["expected"], d["expected"])
    assert np.array_equal(got, golden_stress["expected"]), np.unique(got)


@pytest.mark.parametrize("case", [0, 1])
def test_oracle_qkv_boundary(case, golden_boundary):
    d = synth.qkv_boundary_inputs(case)
    for key in ("x", "q_weight", "k_weight", "v_weight", "q_weight_scale", "input_rms_weight", "kv_offset",
                "rope_offset", "cos_row", "sin_row"):
        assert prng.checksum(d[key]) == int(golden_boundary[f"case{case}.checksum.{key}"][0]), key
    q, k, v = qkv_oracle(d)
    for label, got in (("q", q), ("k", k), ("v", v)):
        want = golden_boundary[f"case{case}.expected.{label}"]
        assert np.array_equal(want, got.reshape(-1)), label


def attention_inputs(golden_attention, case):
    t_len, valid = (int(v) for v in golden_attention[f"case{case}.params"])
    qs = float(golden_attention[f"case{case}.qscale"][0])
    seed = f"golden.attention.case{case}"
    q = prng.bf16_signs(f"{seed}.q", 16 * 256, qs).reshape(8, 2, 256)
    k = prng.bf16_uniform(f"{seed}.k", t_len * 8 * 256, -1.0, 1.0).reshape(t_len, 8, 256)
    v = prng.bf16_uniform(f"{seed}.v", t_len * 8 * 256, -1.0, 1.0).reshape(t_len, 8, 256)
    mask = (np.arange(t_len) < valid).astype(np.float32)
    return q, k, v, mask, qs


@pytest.mark.parametrize("case", range(4))
def test_oracle_attention_vs_reference_sdpa(case, golden_attention):
    """gemma4.py:179-181 computes f32 scores; the device semantics round them to bf16, which at
    |q| = 1 moves scores of magnitude ~30 by up to 2^-3: that case gets the O-op tolerance."""
    q, k, v, mask, qs = attention_inputs(golden_attention, case)
    got = ops.sliding_attention(q, k, v, mask)
    atol = 0.01 if qs < 1.0 else ATOL["sliding_attention_output"]
    ok, maxd, _ = within(golden_attention[f"case{case}.expected"], got, atol)
    assert ok, maxd


def test_attention_oracle_vs_float64(golden_attention):
    q, k, v, mask, _ = attention_inputs(golden_attention, 1)
    got = ops.bf16_to_f32(ops.sliding_attention(q, k, v, mask))
    ref = ops.attention_float64(q, k, v, mask)
    assert np.abs(got - ref).max() < 2e-3


def test_planted_mistake_is_caught(golden_runs):
    """The comparison rule rejects a single wrong element (the mistake is planted in the oracle output)."""
    d = synth.sliding_attention_output(0)
    got = ops.sliding_attention_output(d["x"], d["post_attn_rms_weight"], d["o_weight"], d["o_weight_scale"],
                                       d["residual"]).copy()
    got[1234] = ops.f32_to_bf16(np.array([ops.bf16_to_f32(got[1234:1235])[0] + 0.25], np.float32))[0]
    ok, _, _ = within(golden_runs["run0.sliding_attention_output.expected"], got, ATOL["sliding_attention_output"])
    assert not ok
