"""GPU parity of the global (full-attention) layer ops through the C ABI (FOG/src/ops.rs:78-199)
against the CPU oracle's restatement (oracle/ops.py full_*), on seeded Gaussian inputs: the fused
QKV with the single K = V head and the partial RoPE table, the paged online-softmax attention over
three pages (the last one partly masked, as the current page is), validated also against a float64
softmax, and the output projection with its division by the softmax sum."""

import numpy as np
import pytest

import gaussian
from helpers import ATOL, within
from oracle import ops as oracle
from test_gpu_parity import dev_tensor, host_bits

pytestmark = pytest.mark.gpu
H, GF, DF, QF, TF = 3840, 16, 512, 8192, 512


def test_full_project_qkv(device):
    import torch
    from g4b200 import ops

    r = np.random.default_rng(21)
    pos = 1300
    q_w, q_s = gaussian.fp8_rows(r.standard_normal((QF, H), dtype=np.float32) * np.float32(0.02))
    k_w, k_s = gaussian.fp8_rows(r.standard_normal((DF, H), dtype=np.float32) * np.float32(0.02))
    x = gaussian.bf16(r.standard_normal(H))
    g_in = gaussian.bf16(1 + 0.1 * r.standard_normal(H))
    g_q, g_k = gaussian.bf16(1 + 0.1 * r.standard_normal(DF)), gaussian.bf16(1 + 0.1 * r.standard_normal(DF))
    c, s = oracle.rope_tables(DF, 1e6, 0.25, pos)  # the global table: a quarter of the dims rotate
    cos = np.zeros((2048, DF), np.uint16)
    sin = np.zeros((2048, DF), np.uint16)
    cos[pos], sin[pos] = gaussian.bf16(c), gaussian.bf16(oracle.negate_low_half(s))
    fill_k, fill_v = gaussian.bf16(r.standard_normal((TF, DF))), gaussian.bf16(r.standard_normal((TF, DF)))
    kc, vc = dev_tensor(fill_k), dev_tensor(fill_v)
    qo = torch.zeros((GF, DF), dtype=torch.bfloat16, device="cuda")
    slot = pos % TF
    ops.full_project_qkv(device, dev_tensor(x), dev_tensor(q_w), dev_tensor(k_w), dev_tensor(gaussian.bf16(q_s)),
                         dev_tensor(gaussian.bf16(k_s)), dev_tensor(g_in), dev_tensor(g_q), dev_tensor(g_k),
                         dev_tensor(np.array([slot * DF * 2], np.int32)), dev_tensor(np.array([pos * DF * 2], np.int32)),
                         dev_tensor(cos), dev_tensor(sin), kc, vc, qo)
    device.check()
    wq, wk, wv = oracle.full_project_qkv(x, q_w, k_w, gaussian.bf16(q_s), gaussian.bf16(k_s), g_in, g_q, g_k,
                                         cos[pos], sin[pos])
    k_got, v_got = host_bits(kc), host_bits(vc)
    for want, got in ((wq, host_bits(qo)), (wk, k_got[slot]), (wv, v_got[slot])):
        ok, maxd, exact = within(want, got, ATOL["sliding_project_qkv"])
        assert ok and exact > 0.99, (maxd, exact)
    others = np.ones(TF, bool)
    others[slot] = False
    assert np.array_equal(k_got[others], fill_k[others]) and np.array_equal(v_got[others], fill_v[others])


def test_full_attention_pages(device):
    import torch
    from g4b200 import ops

    r = np.random.default_rng(22)
    q = gaussian.bf16(r.standard_normal((GF, DF)) * 0.05)
    ks = [gaussian.bf16(r.standard_normal((TF, DF))) for _ in range(3)]
    vs = [gaussian.bf16(r.standard_normal((TF, DF))) for _ in range(3)]
    row = 200  # the current page's row: slots past it are masked (the reference's diagonal mask rows)
    masks = [np.ones(TF, np.float32), np.ones(TF, np.float32), (np.arange(TF) <= row).astype(np.float32)]
    rmax = torch.zeros(GF, dtype=torch.float32, device="cuda")
    rsum = torch.zeros_like(rmax)
    out = torch.zeros((GF, DF), dtype=torch.bfloat16, device="cuda")
    m = s = o = None
    qd = dev_tensor(q)
    for p in range(3):
        ops.full_attention_page(device, qd, dev_tensor(ks[p]), dev_tensor(vs[p]), dev_tensor(masks[p]), rmax, rsum,
                                out, first=p == 0)
        device.check()
        m, s, o = oracle.full_attention_page(q, ks[p], vs[p], masks[p], m, s, o) if p else \
            oracle.full_attention_page(q, ks[p], vs[p], masks[p])
        assert np.allclose(rmax.cpu().numpy(), m, rtol=0, atol=0.01), p
        assert np.allclose(rsum.cpu().numpy(), s, rtol=1e-3), p
        ok, maxd, exact = within(o, host_bits(out), 0.01)
        assert ok, (p, maxd)
        assert exact > 0.9, (p, exact)
    y = oracle.bf16_to_f32(host_bits(out)) / rsum.cpu().numpy()[:, None]
    ref = oracle.full_attention_float64(q, ks, vs, masks)
    assert np.abs(y - ref).max() < 0.01 * np.abs(ref).max() + 1e-3


def test_full_attention_output(device):
    import torch
    from g4b200 import ops

    r = np.random.default_rng(23)
    x = gaussian.bf16(r.standard_normal((GF, DF)))
    rsum = (1 + r.random(GF) * 3).astype(np.float32)
    o_w, o_s = gaussian.fp8_rows(r.standard_normal((H, QF), dtype=np.float32) * np.float32(0.02))
    gamma = gaussian.bf16(1 + 0.1 * r.standard_normal(H))
    residual = gaussian.bf16(r.standard_normal(H))
    res = dev_tensor(residual)
    ops.full_attention_output(device, dev_tensor(x), dev_tensor(rsum), dev_tensor(gamma), dev_tensor(o_w),
                              dev_tensor(gaussian.bf16(o_s)), res)
    device.check()
    want = oracle.full_attention_output(x, rsum, gamma, o_w, gaussian.bf16(o_s), residual)
    ok, maxd, exact = within(want, host_bits(res), ATOL["sliding_attention_output"])
    assert ok and exact > 0.99, (maxd, exact)
