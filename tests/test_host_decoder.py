"""CPU: the host side of the decode driver and the FP8 feed-forward (no GPU needed).

- the ctypes mirrors of g4_layer / g4_model (g4b200.decoder) have the C header's layout: a small C
  program compiled with gcc against include/g4b200.h prints every field's offset;
- the decoder entry points refuse a null context;
- the tensor-parallel FP8 FFN oracle (rank-order sum of the down partials) agrees with the
  one-GPU oracle within the reference grader's tolerance, and the Gaussian quantisers of the test
  inputs reproduce their weights within the formats' precision.
"""

import ctypes
import subprocess

import numpy as np
import pytest

from g4b200 import _abi, decoder
from helpers import ATOL, within
from oracle import ops as oracle
import gaussian

INCLUDE = __import__("pathlib").Path(__file__).resolve().parent.parent / "include"


def c_offsets(struct, fields, tmp_path):
    src = tmp_path / "off.c"
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "g4b200.h"', "int main(void) {",
             f'  printf("%zu\\n", sizeof({struct}));']
    lines += [f'  printf("%zu\\n", offsetof({struct}, {f}));' for f in fields]
    lines += ["  return 0;", "}"]
    src.write_text("\n".join(lines))
    exe = tmp_path / "off"
    subprocess.run(["gcc", "-I", str(INCLUDE), str(src), "-o", str(exe)], check=True)
    return [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]


@pytest.mark.parametrize("struct,cls", [("g4_layer", decoder._Layer), ("g4_model", decoder._Model)])
def test_ctypes_mirror_matches_the_header(tmp_path, struct, cls):
    names = [f[0] for f in cls._fields_]
    got = c_offsets(struct, names, tmp_path)
    assert got[0] == ctypes.sizeof(cls)
    assert got[1:] == [getattr(cls, n).offset for n in names]


def test_decoder_entry_points_refuse_a_null_context():
    lib = _abi.lib()
    out = ctypes.c_void_p()
    assert lib.g4_decoder_create(None, None, ctypes.byref(out)) == _abi.G4_ERR_INVALID_ARGUMENT
    assert lib.g4_decoder_step(None, None) == _abi.G4_ERR_INVALID_ARGUMENT
    assert lib.g4_decoder_capture(None, None) == _abi.G4_ERR_INVALID_ARGUMENT
    assert lib.g4_decoder_buffers(None, None, None, None) == _abi.G4_ERR_INVALID_ARGUMENT
    assert lib.g4_decoder_destroy(None) == _abi.G4_ERR_INVALID_ARGUMENT


@pytest.fixture(scope="module")
def ffn8():
    return gaussian.ffn_fp8()


@pytest.mark.parametrize("world", [2, 8])
def test_fp8_ffn_tp_oracle_matches_whole(ffn8, world):
    import torch

    from g4b200 import tp

    d = ffn8
    whole = oracle.feedforward_fp8(d["residual"], d["pre_ff_rms_weight"], d["up_weight"], d["gate_weight"],
                                   d["down_weight"], d["up_weight_scale"], d["gate_weight_scale"],
                                   d["down_weight_scale"], d["post_ff_rms_weight"], d["layer_scalar"])

    def cut(name, arr, r):
        return tp.shard(name, torch.from_numpy(arr), r, world).numpy()

    up = [(cut("up_weight", d["up_weight"], r), cut("up_channel_scale", d["up_weight_scale"], r)) for r in range(world)]
    gate = [(cut("gate_weight", d["gate_weight"], r), cut("gate_channel_scale", d["gate_weight_scale"], r))
            for r in range(world)]
    down = [cut("down_weight", d["down_weight"], r) for r in range(world)]
    assert down[0].shape[1] == (2048 if world == 8 else 15360 // world)  # zero-padded to whole units
    parts = oracle.feedforward_fp8_tp(d["residual"], d["pre_ff_rms_weight"], up, gate, down, d["down_weight_scale"],
                                      d["post_ff_rms_weight"], d["layer_scalar"])
    ok, maxd, exact = within(whole, parts, ATOL["decoder_feedforward"])
    assert ok and exact > 0.95, (maxd, exact)


def test_gaussian_quantisers_reproduce_their_weights():
    r = np.random.default_rng(3)
    w = r.standard_normal((64, 512), dtype=np.float32) * np.float32(0.02)
    codes, scale = gaussian.fp8_rows(w)
    back = oracle.e4m3_to_f32(codes) * scale[:, None]
    assert np.all(np.abs(back - w) <= np.abs(w) * 2.0 ** -4 + scale[:, None] * 2.0 ** -9)
    packed, bscale, g = gaussian.nvfp4(w)
    back = oracle.nvfp4_dequant(packed, bscale, 64, 512) * g[0]
    blk = np.abs(w).reshape(64, 32, 16).max(axis=2, keepdims=True)
    err = np.abs(back - w).reshape(64, 32, 16)
    assert np.all(err <= blk * 0.3)  # e2m1: a step of at most 1/4 of the block's largest value (and scale rounding)
