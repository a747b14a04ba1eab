"""CPU: the batched feed-forward oracles are the single-token reference ops applied row by row
(FOG/src/ops.rs:201-239 per token), for both weight formats (small shapes: the oracle functions
take the hidden and intermediate sizes)."""

import numpy as np

import gaussian
from oracle import ops as oracle

HID, INTER = 256, 512


def _rows(seed, n=3):
    return gaussian.bf16(np.random.default_rng(seed).standard_normal((n, HID)))


def test_nvfp4_batch_oracle_is_row_by_row():
    r = np.random.default_rng(11)
    d = {}
    for name, shape in (("up", (INTER, HID)), ("gate", (INTER, HID)), ("down", (HID, INTER))):
        d[name] = gaussian.nvfp4(r.standard_normal(shape, dtype=np.float32) * np.float32(0.02))
    pre, post = gaussian.bf16(1 + 0.1 * r.standard_normal(HID)), gaussian.bf16(1 + 0.1 * r.standard_normal(HID))
    ls = gaussian.bf16(np.full(8, 0.375))
    args = (pre, d["up"][0], d["gate"][0], d["down"][0], d["up"][1], d["gate"][1], d["down"][1], d["up"][2][0],
            d["gate"][2][0], d["down"][2][0], post, ls)
    rows = _rows(1)
    got = oracle.decoder_feedforward_batch(rows, *args, hidden=HID, inter=INTER)
    for i in range(len(rows)):
        assert np.array_equal(got[i], oracle.decoder_feedforward(rows[i], *args, hidden=HID, inter=INTER))


def test_fp8_batch_oracle_is_row_by_row():
    r = np.random.default_rng(12)
    up, up_s = gaussian.fp8_rows(r.standard_normal((INTER, HID), dtype=np.float32) * np.float32(0.02))
    gate, gate_s = gaussian.fp8_rows(r.standard_normal((INTER, HID), dtype=np.float32) * np.float32(0.02))
    down, down_s = gaussian.fp8_rows(r.standard_normal((HID, INTER), dtype=np.float32) * np.float32(0.02))
    pre, post = gaussian.bf16(1 + 0.1 * r.standard_normal(HID)), gaussian.bf16(1 + 0.1 * r.standard_normal(HID))
    args = (pre, up, gate, down, up_s, gate_s, down_s, post, gaussian.bf16(np.full(8, 0.375)))
    rows = _rows(2)
    got = oracle.feedforward_fp8_batch(rows, *args, hidden=HID, inter=INTER)
    for i in range(len(rows)):
        assert np.array_equal(got[i], oracle.feedforward_fp8(rows[i], *args, hidden=HID, inter=INTER))
