"""GPU: g4_sliding_attention_output_noalloc (no context, static scratch) through the C ABI.

It must give what g4_sliding_attention_output gives on the same inputs, call after call: two
calls in a row update the residual in place twice, and each result is compared with the
context-based entry point's result at the same step. Both launch the same kernel with the same
fixed summation order, so the results must be identical bit for bit (a stale word or a missed
clear of the static block would show up as a difference); the oracle tolerance of the reference
grader applies only to the comparison with the reference's expected output. The file name sorts
last so the check also runs after every other GPU test.
"""

import ctypes

import numpy as np
import pytest

from oracle import synth
from helpers import ATOL, within

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_matches_context_entry_point_twice(device, golden_runs):
    import torch

    from g4b200 import _abi, ops

    d = synth.sliding_attention_output(0)

    def dev(arr):
        a = np.ascontiguousarray(arr)
        t = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()
        return t.view(torch.bfloat16) if a.dtype == np.uint16 else t

    def bits(t):
        return t.cpu().view(torch.int16).numpy().view(np.uint16)

    x, gamma, w, s = dev(d["x"]), dev(d["post_attn_rms_weight"]), dev(d["o_weight"]), dev(d["o_weight_scale"])
    res_ctx = dev(d["residual"])
    res_static = dev(d["residual"])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    lib = _abi.lib()
    for step in range(2):
        ops.sliding_attention_output(device, x, gamma, w, s, res_ctx)
        st = lib.g4_sliding_attention_output_noalloc(_ptr(x), _ptr(gamma), _ptr(w), _ptr(s), _ptr(res_static), stream)
        assert st == _abi.G4_OK, lib.g4_status_string(st).decode()
        torch.cuda.synchronize()
        device.check()
        got, want = bits(res_static), bits(res_ctx)
        assert np.array_equal(got, want), (step, int(np.sum(got != want)))
        if step == 0:  # one call on the reference's run-0 inputs: the grader's tolerance holds
            ok, maxd, _ = within(golden_runs["run0.sliding_attention_output.expected"], got,
                                 ATOL["sliding_attention_output"])
            assert ok, maxd


def test_noalloc_rejects_bad_pointers(device):
    import torch

    from g4b200 import _abi

    lib = _abi.lib()
    buf = torch.zeros(8192, dtype=torch.uint8, device="cuda")
    p = ctypes.c_void_p(buf.data_ptr())
    odd = ctypes.c_void_p(buf.data_ptr() + 8)
    assert lib.g4_sliding_attention_output_noalloc(None, p, p, p, p, None) == _abi.G4_ERR_INVALID_ARGUMENT
    assert lib.g4_sliding_attention_output_noalloc(p, p, odd, p, p, None) == _abi.G4_ERR_MISALIGNED
