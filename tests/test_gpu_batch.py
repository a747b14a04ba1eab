"""GPU parity of the token-batched NVFP4 feed-forward (BASELINE configs[3]'s M sweep) through the C
ABI: g4_decoder_feedforward_batch on M residual rows against the oracle run row by row
(oracle.decoder_feedforward_batch, the reference op FOG/src/ops.rs:201-239 per token), on
BASELINE's Gaussian distributions and on the reference's own seeded inputs, whose golden outputs
every row of a batch of copies must reproduce. Tolerance: the reference grader's
(FOG/src/bin/test_kernels.rs:447-465)."""

import numpy as np
import pytest

import gaussian
from helpers import ATOL, within
from oracle import ops as oracle
from oracle import synth
from test_gpu_parity import dev_tensor, host_bits, run_ffn

pytestmark = pytest.mark.gpu

WEIGHTS = ("up_weight_packed", "gate_weight_packed", "down_weight_packed", "up_weight_scale", "gate_weight_scale",
           "down_weight_scale", "up_global_scale", "gate_global_scale", "down_global_scale")


def run_batch(device, d, residual, tiled=False):
    from g4b200 import ops

    res = dev_tensor(np.ascontiguousarray(residual))
    w = {k: dev_tensor(d[k]) for k in WEIGHTS}
    tail = [w["up_global_scale"], w["gate_global_scale"], w["down_global_scale"], dev_tensor(d["post_ff_rms_weight"]),
            dev_tensor(d["layer_scalar"])]
    if tiled:
        ug = ops.pack_upgate(device, w["up_weight_packed"], w["gate_weight_packed"], scales=False)
        ugs = ops.pack_upgate(device, w["up_weight_scale"], w["gate_weight_scale"], scales=True)
        dn = ops.tile_weight(device, "down_weight_packed", w["down_weight_packed"])
        dns = ops.tile_weight(device, "down_weight_scale", w["down_weight_scale"])
        ops.decoder_feedforward_batch_tiled(device, res, dev_tensor(d["pre_ff_rms_weight"]), ug, dn, ugs, dns, *tail)
    else:
        ops.decoder_feedforward_batch(device, res, dev_tensor(d["pre_ff_rms_weight"]), w["up_weight_packed"],
                                      w["gate_weight_packed"], w["down_weight_packed"], w["up_weight_scale"],
                                      w["gate_weight_scale"], w["down_weight_scale"], *tail)
    device.check()
    return host_bits(res)


def oracle_batch(d, residual):
    return oracle.decoder_feedforward_batch(residual, d["pre_ff_rms_weight"], *(d[k] for k in WEIGHTS[:6]),
                                            d["up_global_scale"][0], d["gate_global_scale"][0],
                                            d["down_global_scale"][0], d["post_ff_rms_weight"], d["layer_scalar"])


@pytest.fixture(scope="module")
def gauss():
    d = gaussian.ffn_nvfp4()
    rows = gaussian.bf16(np.random.default_rng(3064).standard_normal((64, 3840)))
    return d, rows, oracle_batch(d, rows)


@pytest.mark.parametrize("m", [2, 8, 16, 17, 33, 64])
def test_batch_matches_oracle_row_by_row(device, gauss, m):
    """M tokens of N(0,1) activations on N(0, 0.02) NVFP4 weights."""
    d, rows, want = gauss
    got = run_batch(device, d, rows[:m])
    for i in range(m):
        ok, maxd, exact = within(want[i], got[i], ATOL["decoder_feedforward"])
        assert ok, (m, i, maxd)
        assert exact > 0.95, (m, i, exact)


def test_batch_deterministic_and_tiled_identical(device, gauss):
    d, rows, _ = gauss
    got = run_batch(device, d, rows[:48])
    assert np.array_equal(run_batch(device, d, rows[:48]), got)
    assert np.array_equal(run_batch(device, d, rows[:48], tiled=True), got)


def test_batch_rows_independent(device, gauss):
    """A row's result does not depend on the other rows of its batch or on the batch size."""
    d, rows, _ = gauss
    full = run_batch(device, d, rows[:64])
    part = run_batch(device, d, rows[5:21])
    assert np.array_equal(full[5:21], part)


def test_batch_of_one_is_the_single_token_op(device, gauss):
    d, rows, _ = gauss
    assert np.array_equal(run_batch(device, d, rows[:1]), run_ffn(device, dict(d, residual=rows[0])).reshape(1, -1))


@pytest.mark.parametrize("run", [0, 4, 8])
def test_batch_reproduces_the_reference_outputs(device, run, golden_runs):
    """The reference's seeded FFN inputs (runs of generate_references.py): every row of a batch of
    16 copies matches the reference's golden output, and all rows are identical."""
    d = synth.decoder_feedforward(run)
    got = run_batch(device, d, np.tile(d["residual"].reshape(1, -1), (16, 1)))
    want = golden_runs[f"run{run}.decoder_feedforward.expected"]
    assert all(np.array_equal(got[0], got[i]) for i in range(16))
    ok, maxd, exact = within(want, got[0], ATOL["decoder_feedforward"])
    assert ok, maxd
    assert exact > 0.95, exact


def test_batch_stress_case(device, golden_stress):
    """The correlated FFN-stress input (every output bf16 0x3ecf) in a batch of 8."""
    d = synth.ffn_stress()
    got = run_batch(device, d, np.tile(d["residual"].reshape(1, -1), (8, 1)))
    for i in range(8):
        ok, maxd, exact = within(golden_stress["expected"], got[i], ATOL["decoder_feedforward"])
        assert ok, (i, maxd)


def test_batch_zero_rows(device, gauss):
    d, rows, _ = gauss
    z = rows[:8].copy()
    z[3] = 0
    got = run_batch(device, d, z)
    want = oracle_batch(d, z)
    for i in range(8):
        assert within(want[i], got[i], ATOL["decoder_feedforward"])[0], i


def test_batch_rejects_bad_sizes(device, gauss):
    from g4b200 import ops

    d, rows, _ = gauss
    with pytest.raises(ValueError):
        run_batch(device, d, np.zeros((65, 3840), np.uint16))
    with pytest.raises(ValueError):
        ops.decoder_feedforward_batch(device, dev_tensor(rows[0]), *([None] * 12))


# --- FP8 weights with f32 per-row scales (BASELINE configs[0]'s format, batched)

FP8_WEIGHTS = ("up_weight", "gate_weight", "down_weight", "up_weight_scale", "gate_weight_scale", "down_weight_scale")


def run_batch8(device, d, residual, tiled=False):
    from g4b200 import ops

    res = dev_tensor(np.ascontiguousarray(residual))
    w = {k: dev_tensor(d[k]) for k in FP8_WEIGHTS}
    tail = [w["up_weight_scale"], w["gate_weight_scale"], w["down_weight_scale"], dev_tensor(d["post_ff_rms_weight"]),
            dev_tensor(d["layer_scalar"])]
    if tiled:
        ug = ops.pack_upgate_fp8(device, w["up_weight"], w["gate_weight"])
        dn = ops.tile_weight(device, "down_weight", w["down_weight"])
        ops.decoder_feedforward_fp8_batch_tiled(device, res, dev_tensor(d["pre_ff_rms_weight"]), ug, dn, *tail)
    else:
        ops.decoder_feedforward_fp8_batch(device, res, dev_tensor(d["pre_ff_rms_weight"]), w["up_weight"],
                                          w["gate_weight"], w["down_weight"], *tail)
    device.check()
    return host_bits(res)


@pytest.fixture(scope="module")
def gauss8():
    d = gaussian.ffn_fp8()
    rows = gaussian.bf16(np.random.default_rng(3065).standard_normal((64, 3840)))
    want = oracle.feedforward_fp8_batch(rows, d["pre_ff_rms_weight"], *(d[k] for k in FP8_WEIGHTS),
                                        d["post_ff_rms_weight"], d["layer_scalar"])
    return d, rows, want


@pytest.mark.parametrize("m", [2, 16, 17, 32, 33, 64])
def test_fp8_batch_matches_oracle_row_by_row(device, gauss8, m):
    """configs[0]'s FP8 FFN on M tokens of N(0,1) activations."""
    d, rows, want = gauss8
    got = run_batch8(device, d, rows[:m])
    for i in range(m):
        ok, maxd, exact = within(want[i], got[i], ATOL["decoder_feedforward"])
        assert ok, (m, i, maxd)
        assert exact > 0.95, (m, i, exact)


def test_fp8_batch_tiled_identical_and_rows_independent(device, gauss8):
    """Both engines (kind::f16 tiles above 16 tokens, e4m3 term operands up to 16): the unit-tiled
    weights give the same bits, and a token's result does not depend on the batch it came in
    within an engine; across the engines the results agree within the tolerance."""
    from helpers import within

    d, rows, _ = gauss8
    got = run_batch8(device, d, rows[:40])
    assert np.array_equal(run_batch8(device, d, rows[:40], tiled=True), got)
    assert np.array_equal(run_batch8(device, d, rows[3:20]), got[3:20])
    small = run_batch8(device, d, rows[:16])
    assert np.array_equal(run_batch8(device, d, rows[:16], tiled=True), small)
    assert np.array_equal(run_batch8(device, d, rows[3:9]), small[3:9])
    ok, maxd, _ = within(got[:16].reshape(-1), small.reshape(-1), 0.01)
    assert ok, maxd


def test_fp8_batch_of_one_is_the_single_token_op(device, gauss8):
    from test_gpu_gaussian import run_ffn_fp8

    d, rows, _ = gauss8
    assert np.array_equal(run_batch8(device, d, rows[:1]), run_ffn_fp8(device, dict(d, residual=rows[0])).reshape(1, -1))
