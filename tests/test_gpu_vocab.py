"""GPU parity of the vocabulary ends through the C ABI: embed_token (FOG/src/ops.rs:8-35) and
final_norm_and_logits (FOG/src/ops.rs:241-298) against the CPU oracle's restatement of the device
ops, on seeded Gaussian tables (the reference ties the lm_head to the embedding table)."""

import numpy as np
import pytest

from helpers import within
from oracle import ops as oracle
from test_gpu_parity import dev_tensor, host_bits

pytestmark = pytest.mark.gpu
H = 3840


def table(rows, seed):
    r = np.random.default_rng(seed)
    return oracle.f32_to_bf16((r.standard_normal((rows, H), dtype=np.float32) * np.float32(0.03)))


def run_logits(device, x, gamma, tab):
    import torch
    from g4b200 import ops

    out = torch.zeros(tab.shape[0], dtype=torch.bfloat16, device="cuda")
    ops.final_norm_and_logits(device, dev_tensor(x), dev_tensor(gamma), dev_tensor(tab), out)
    device.check()
    return host_bits(out)


def test_embed_token_exact(device):
    import torch
    from g4b200 import ops

    tab = table(4096, 1)
    for token in (0, 1234, 4095):
        out = torch.zeros(H, dtype=torch.bfloat16, device="cuda")
        ops.embed_token(device, dev_tensor(tab), dev_tensor(np.array([token * H * 2], np.int32)), out)
        device.check()
        assert np.array_equal(host_bits(out), oracle.embed_token(tab, token)), token


def test_embed_token_bad_offset(device):
    import torch
    from g4b200 import G4Error, ops

    tab = table(256, 2)
    out = torch.zeros(H, dtype=torch.bfloat16, device="cuda")
    for off in (256 * H * 2, 3, -2 * H):  # one row past the table, misaligned, negative
        with pytest.raises(G4Error) as err:
            ops.embed_token(device, dev_tensor(tab), dev_tensor(np.array([off], np.int32)), out)
            device.check()
        assert err.value.flags & 64


def test_logits_match_oracle(device):
    r = np.random.default_rng(5)
    x = oracle.f32_to_bf16(r.standard_normal(H, dtype=np.float32))
    gamma = oracle.f32_to_bf16(1 + 0.1 * r.standard_normal(H).astype(np.float32))
    tab = table(16384, 3)
    got = run_logits(device, x, gamma, tab)
    ok, maxd, exact = within(oracle.final_norm_and_logits(x, gamma, tab), got, 0.01)
    assert ok, maxd
    assert exact > 0.95, exact


def test_logits_row_slice_is_a_tensor_parallel_rank(device):
    """A rank passing rows [a, b) of the table gets exactly those rows' logits."""
    r = np.random.default_rng(6)
    x = oracle.f32_to_bf16(r.standard_normal(H, dtype=np.float32))
    gamma = oracle.f32_to_bf16(np.ones(H, np.float32))
    tab = table(8192, 4)
    whole = run_logits(device, x, gamma, tab)
    part = run_logits(device, x, gamma, np.ascontiguousarray(tab[3000:5048]))
    assert np.array_equal(part, whole[3000:5048])


def test_logits_full_vocabulary(device):
    """The reference's W = 262144 rows (2 GB): a strided sample of rows against the oracle."""
    import torch
    from g4b200 import ops

    r = np.random.default_rng(7)
    x = oracle.f32_to_bf16(r.standard_normal(H, dtype=np.float32))
    gamma = oracle.f32_to_bf16(1 + 0.1 * r.standard_normal(H).astype(np.float32))
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    tab = (torch.randn((262144, H), generator=g, device="cuda") * 0.03).to(torch.bfloat16)
    out = torch.zeros(262144, dtype=torch.bfloat16, device="cuda")
    ops.final_norm_and_logits(device, dev_tensor(x), dev_tensor(gamma), tab, out)
    device.check()
    rows = np.arange(0, 262144, 97)
    sample = host_bits(tab[torch.from_numpy(rows).cuda()])
    ok, maxd, exact = within(oracle.final_norm_and_logits(x, gamma, sample), host_bits(out)[rows], 0.01)
    assert ok, maxd
    assert exact > 0.95, exact
