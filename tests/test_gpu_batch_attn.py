"""GPU parity of the batched attention block (g4_sliding_project_qkv_batch, g4_sliding_attention_batch,
g4_sliding_attention_output_batch): m sequences, each with its own ring cache and position, against the
single-token oracle ops applied sequence by sequence (FOG/src/ops.rs:37-76, 118-146; oracle
generate_references.py:321-334, 353-355), on BASELINE configs[1]/[2]'s Gaussian distributions.
Tolerances are the reference grader's (FOG/src/bin/test_kernels.rs:447-465); attention is held to
0.01 as in tests/test_gpu_gaussian.py."""

import numpy as np
import pytest

import gaussian
from helpers import ATOL, within
from oracle import ops as oracle
from oracle.ops import negate_low_half, rope_tables
from test_gpu_parity import dev_tensor, host_bits

pytestmark = pytest.mark.gpu

NS, GS, DS, H, QS = 8, 2, 256, 3840, 4096
ROPE_ROWS = 4096


def qkv_batch_inputs(m, ring, theta, seed):
    """Shared QKV weights, m token rows, m distinct positions, m rings."""
    d = gaussian.qkv(theta, ring=ring, salt=seed)
    r = np.random.default_rng(500 + seed)
    d["xs"] = gaussian.bf16(r.standard_normal((m, H)))
    d["positions"] = r.choice(ROPE_ROWS, size=m, replace=False)
    cos = np.zeros((ROPE_ROWS, DS), np.uint16)
    sin = np.zeros((ROPE_ROWS, DS), np.uint16)
    for p in d["positions"]:
        c, s = rope_tables(DS, theta, 1.0, int(p))
        cos[p], sin[p] = gaussian.bf16(c), gaussian.bf16(negate_low_half(s))
    d["cos"], d["sin"] = cos, sin
    d["kv_offsets"] = np.array([(p % ring) * NS * DS * 2 for p in d["positions"]], np.int32)
    d["rope_offsets"] = np.array([p * DS * 2 for p in d["positions"]], np.int32)
    d["k_caches"] = gaussian.bf16(r.standard_normal((m, ring, NS, DS)))
    d["v_caches"] = gaussian.bf16(r.standard_normal((m, ring, NS, DS)))
    return d


def run_qkv_batch(device, d, m=None, tiled=False, keep=None):
    """The batched QKV op on the first m sequences of `d`: (q_out, k caches, v caches) as bits.
    `keep` (a list) receives the device tensors before the error check."""
    from g4b200 import ops

    m = len(d["xs"]) if m is None else m
    kc, vc = dev_tensor(d["k_caches"][:m]), dev_tensor(d["v_caches"][:m])
    qo = dev_tensor(np.zeros((m, NS, GS, DS), np.uint16))
    names = ("q_weight", "k_weight", "v_weight")
    if tiled:
        w = [ops.tile_weight(device, n, dev_tensor(d[n])) for n in names]
    else:
        w = [dev_tensor(d[n]) for n in names]
    ops.sliding_project_qkv_batch(
        device, dev_tensor(d["xs"][:m]), *w,
        *(dev_tensor(d[k]) for k in ("q_weight_scale", "k_weight_scale", "v_weight_scale", "input_rms_weight",
                                     "q_rms_weight", "k_rms_weight")),
        dev_tensor(d["kv_offsets"][:m]), dev_tensor(d["rope_offsets"][:m]), dev_tensor(d["cos"]), dev_tensor(d["sin"]),
        kc, vc, qo, tiled=tiled)
    if keep is not None:
        keep.extend((qo, kc, vc))
    device.check()
    return host_bits(qo), host_bits(kc), host_bits(vc)


@pytest.mark.parametrize("m", [2, 8, 17, 32, 33])
def test_qkv_batch_matches_oracle_per_sequence(device, m):
    """Each sequence's q, its K / V slot, and every other slot of every ring untouched."""
    ring = 1024
    d = qkv_batch_inputs(m, ring, 1e4, seed=m)
    q, kc, vc = run_qkv_batch(device, d)
    for i in range(m):
        p = int(d["positions"][i])
        wq, wk, wv = oracle.sliding_project_qkv(d["xs"][i], d["q_weight"], d["k_weight"], d["v_weight"],
                                                d["q_weight_scale"], d["k_weight_scale"], d["v_weight_scale"],
                                                d["input_rms_weight"], d["q_rms_weight"], d["k_rms_weight"],
                                                d["cos"][p], d["sin"][p])
        slot = p % ring
        for want, got in ((wq, q[i]), (wk, kc[i, slot]), (wv, vc[i, slot])):
            ok, maxd, exact = within(want, got, ATOL["sliding_project_qkv"])
            assert ok and exact > 0.99, (i, maxd, exact)
        others = np.ones(ring, bool)
        others[slot] = False
        assert np.array_equal(kc[i][others], d["k_caches"][i][others])
        assert np.array_equal(vc[i][others], d["v_caches"][i][others])


def test_qkv_batch_tiled_identical_and_batch_independent(device):
    """For both engines (kind::f16 tiles above 16 sequences, e4m3 term operands up to 16): the
    unit-tiled weights give the same bits, and a sequence's result does not depend on the batch it
    came in (33 vs 17 sequences, 16 vs 2)."""
    d = qkv_batch_inputs(33, 1024, 1e6, seed=7)
    for big, small in ((33, 17), (16, 2)):
        q, kc, vc = run_qkv_batch(device, d, m=big)
        qt, kct, vct = run_qkv_batch(device, d, m=big, tiled=True)
        assert np.array_equal(q, qt) and np.array_equal(kc, kct) and np.array_equal(vc, vct)
        q2, kc2, vc2 = run_qkv_batch(device, d, m=small)
        assert np.array_equal(q2, q[:small]) and np.array_equal(kc2, kc[:small])
        assert np.array_equal(vc2, vc[:small])


def test_qkv_batch_bad_offset_skips_only_that_sequence(device):
    """A kv_offset outside the ring raises the device's kv-offset bit (bit 0); that sequence's
    stores are skipped, the others are those of a clean call."""
    from g4b200 import G4Error

    d = qkv_batch_inputs(4, 1024, 1e4, seed=3)
    q_ok, kc_ok, vc_ok = run_qkv_batch(device, d)
    bad = dict(d)
    bad["kv_offsets"] = d["kv_offsets"].copy()
    bad["kv_offsets"][2] = 1024 * NS * DS * 2  # one slot past the ring
    kept = []
    with pytest.raises(G4Error) as err:
        run_qkv_batch(device, bad, keep=kept)
    assert err.value.flags & 1
    q, kc, vc = (host_bits(t) for t in kept)
    for i in (0, 1, 3):
        assert np.array_equal(q[i], q_ok[i]) and np.array_equal(kc[i], kc_ok[i]) and np.array_equal(vc[i], vc_ok[i])
    assert np.array_equal(kc[2], d["k_caches"][2]) and np.array_equal(vc[2], d["v_caches"][2])
    assert not q[2].any()  # q_out starts zeroed


def attention_batch_inputs(m, ring, seed):
    r = np.random.default_rng(900 + seed)
    q = gaussian.bf16(r.standard_normal((m, NS, GS, DS)))
    k = gaussian.bf16(r.standard_normal((m, ring, NS, DS)))
    v = gaussian.bf16(r.standard_normal((m, ring, NS, DS)))
    valid = r.integers(ring // 4, ring + 1, size=m)  # a different fill per sequence
    mask = (np.arange(ring)[None, :] < valid[:, None]).astype(np.float32)
    return q, k, v, mask


@pytest.mark.parametrize("ring,m", [(1024, 3), (4096, 3), (1024, 17), (4096, 17)])
def test_attention_batch_is_the_single_op_per_sequence(device, ring, m):
    """Each sequence within 0.01 of the oracle and of g4_sliding_attention on it alone (a batch splits
    each head's ring over 4 CTAs instead of 8: the partial sums are added in another order)."""
    import torch
    from g4b200 import ops

    q, k, v, mask = attention_batch_inputs(m, ring, ring + m)
    out = torch.zeros((m, NS, GS, DS), dtype=torch.bfloat16, device="cuda")
    ops.sliding_attention_batch(device, dev_tensor(q), dev_tensor(k), dev_tensor(v), dev_tensor(mask), out,
                                scale=1.0 / 16)
    device.check()
    got = host_bits(out)
    for i in range(m):
        one = torch.zeros((NS, GS, DS), dtype=torch.bfloat16, device="cuda")
        ops.sliding_attention(device, dev_tensor(q[i]), dev_tensor(k[i]), dev_tensor(v[i]), dev_tensor(mask[i]), one,
                              scale=1.0 / 16)
        device.check()
        ok, maxd, exact = within(host_bits(one), got[i], 0.01)
        assert ok and exact > 0.95, (i, maxd, exact)
        ok, maxd, exact = within(oracle.sliding_attention(q[i], k[i], v[i], mask[i], 1.0 / 16), got[i], 0.01)
        assert ok and exact > 0.9, (i, maxd, exact)


def test_attention_batch_after_qkv_batch(device):
    """The decoder's order: the batched QKV op, then the batched attention given its kv_offset
    (the early copies may not miss any sequence's new slot): bit-identical to the attention
    without the offsets on the updated caches."""
    import torch
    from g4b200 import ops

    m, ring = 5, 1024
    d = qkv_batch_inputs(m, ring, 1e4, seed=11)
    kc, vc = dev_tensor(d["k_caches"]), dev_tensor(d["v_caches"])
    qo = dev_tensor(np.zeros((m, NS, GS, DS), np.uint16))
    kv = dev_tensor(d["kv_offsets"])
    mask = np.stack([(np.arange(ring) <= min(int(p), ring - 1)).astype(np.float32) for p in d["positions"]])
    fast = torch.zeros((m, NS, GS, DS), dtype=torch.bfloat16, device="cuda")
    plain = torch.zeros_like(fast)
    device.set_overlap(True)
    try:
        ops.sliding_project_qkv_batch(
            device, dev_tensor(d["xs"]),
            *(dev_tensor(d[k]) for k in ("q_weight", "k_weight", "v_weight", "q_weight_scale", "k_weight_scale",
                                         "v_weight_scale", "input_rms_weight", "q_rms_weight", "k_rms_weight")),
            kv, dev_tensor(d["rope_offsets"]), dev_tensor(d["cos"]), dev_tensor(d["sin"]), kc, vc, qo)
        ops.sliding_attention_batch(device, qo, kc, vc, dev_tensor(mask), fast, scale=1.0 / 16, kv_offset=kv)
        ops.sliding_attention_batch(device, qo, kc, vc, dev_tensor(mask), plain, scale=1.0 / 16)
        device.check()
    finally:
        device.set_overlap(False)
    assert np.array_equal(host_bits(fast), host_bits(plain))


def o_batch_inputs(m, seed):
    d = gaussian.attention_output(salt=seed)
    r = np.random.default_rng(700 + seed)
    d["xs"] = gaussian.bf16(r.standard_normal((m, NS, GS, DS)))
    d["residuals"] = gaussian.bf16(r.standard_normal((m, H)))
    return d


def run_o_batch(device, d, m=None, tiled=False):
    from g4b200 import ops

    m = len(d["xs"]) if m is None else m
    res = dev_tensor(d["residuals"][:m])
    w = ops.tile_weight(device, "o_weight", dev_tensor(d["o_weight"])) if tiled else dev_tensor(d["o_weight"])
    ops.sliding_attention_output_batch(device, dev_tensor(d["xs"][:m]), dev_tensor(d["post_attn_rms_weight"]), w,
                                       dev_tensor(d["o_weight_scale"]), res, tiled=tiled)
    device.check()
    return host_bits(res)


@pytest.mark.parametrize("m", [2, 16, 17, 32, 64])
def test_o_batch_matches_oracle_per_sequence(device, m):
    d = o_batch_inputs(m, seed=m)
    got = run_o_batch(device, d)
    for i in range(m):
        want = oracle.sliding_attention_output(d["xs"][i], d["post_attn_rms_weight"], d["o_weight"],
                                               d["o_weight_scale"], d["residuals"][i])
        ok, maxd, exact = within(want, got[i], ATOL["sliding_attention_output"])
        assert ok and exact > 0.99, (i, maxd, exact)


def test_o_batch_tiled_identical_and_batch_independent(device):
    d = o_batch_inputs(40, seed=5)
    for big, small in ((40, 20), (16, 3)):  # each engine
        got = run_o_batch(device, d, m=big)
        assert np.array_equal(run_o_batch(device, d, m=big, tiled=True), got)
        assert np.array_equal(run_o_batch(device, d, m=small), got[:small])
