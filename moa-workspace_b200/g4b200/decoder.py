"""Host mirror of the decode driver (include/g4b200.h, g4_decoder_*): one token through a whole
model per call, the role of the reference host's Decode::run / run_layers
(furiosa-opt-gemma4-12B/src/host/runtime.rs:340-451).

A model is a list of `Layer`s (torch tensors on the device: this rank's slices on a
tensor-parallel device) plus the optional embedding table, final norm and lm_head, and the RoPE
tables. `Decoder.step(token, position)` writes the two device-resident inputs and runs one step;
`Decoder.capture()` records a step as a CUDA graph that later steps replay.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, fields

import torch

from . import _abi
from .ops import Device, _check, _stream_ptr

LAYER_SLIDING, LAYER_FULL = 0, 1
ROPE_LOCAL, ROPE_GLOBAL = 0, 1
FFN_NVFP4, FFN_FP8 = 0, 1


class _Layer(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("rope", ctypes.c_int32), ("ring_len", ctypes.c_int32),
                ("ffn", ctypes.c_int32),
                ("tiled", ctypes.c_int32), ("attn_scale", ctypes.c_float)] + [
        (name, ctypes.c_void_p) for name in (
            "input_rms_weight", "q_weight", "k_weight", "v_weight", "q_weight_scale", "k_weight_scale",
            "v_weight_scale", "q_rms_weight", "k_rms_weight", "k_cache", "v_cache", "post_attn_rms_weight",
            "o_weight", "o_weight_scale", "pre_ff_rms_weight", "post_ff_rms_weight", "layer_scalar", "up_weight",
            "gate_weight", "down_weight", "up_scale", "gate_scale", "down_scale", "up_global_scale",
            "gate_global_scale", "down_global_scale")]


class _Model(ctypes.Structure):
    _fields_ = [("layers", ctypes.POINTER(_Layer)), ("n_layers", ctypes.c_int32),
                ("embedding_table", ctypes.c_void_p), ("vocab_rows", ctypes.c_int32),
                ("final_norm_weight", ctypes.c_void_p), ("lm_head_weight", ctypes.c_void_p),
                ("lm_head_rows", ctypes.c_int32), ("cos_local", ctypes.c_void_p), ("sin_local", ctypes.c_void_p),
                ("cos_global", ctypes.c_void_p), ("sin_global", ctypes.c_void_p), ("rope_rows", ctypes.c_int32),
                ("cos_full", ctypes.c_void_p), ("sin_full", ctypes.c_void_p)]


@dataclass
class Layer:
    """One decoder layer: the tensors of the four op calls (names of the g4_layer fields). For an
    NVFP4 feed-forward up/gate/down_scale are the e4m3 block scales and *_global_scale the f32
    multipliers; for FP8 they are the f32 channel scales. tiled=True: the g4_pack_tiles layout
    (up_weight / up_scale then hold the interleaved up|gate buffers)."""
    input_rms_weight: torch.Tensor
    q_weight: torch.Tensor
    k_weight: torch.Tensor
    v_weight: torch.Tensor | None
    q_weight_scale: torch.Tensor
    k_weight_scale: torch.Tensor
    v_weight_scale: torch.Tensor | None
    q_rms_weight: torch.Tensor
    k_rms_weight: torch.Tensor
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    post_attn_rms_weight: torch.Tensor
    o_weight: torch.Tensor
    o_weight_scale: torch.Tensor
    pre_ff_rms_weight: torch.Tensor
    post_ff_rms_weight: torch.Tensor
    layer_scalar: torch.Tensor
    up_weight: torch.Tensor
    gate_weight: torch.Tensor | None
    down_weight: torch.Tensor
    up_scale: torch.Tensor
    gate_scale: torch.Tensor | None
    down_scale: torch.Tensor
    up_global_scale: torch.Tensor | None = None
    gate_global_scale: torch.Tensor | None = None
    down_global_scale: torch.Tensor | None = None
    rope: int = ROPE_LOCAL
    ffn: int = FFN_NVFP4
    kind: int = LAYER_SLIDING
    tiled: bool = False
    attn_scale: float = 1.0

    @property
    def ring_len(self) -> int:
        """KV slots: a sliding ring [slots, Ns, Ds] (a batched decoder's [batch, slots, Ns, Ds]), or a
        full layer's pages [slots, Df]."""
        return self.k_cache.shape[1] if self.k_cache.dim() == 4 else self.k_cache.shape[0]


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p()


class Decoder:
    """g4_decoder over `layers` on `device` (an ops.Device). The tensors must stay alive as long
    as the decoder does (it keeps references).

    batch > 1 (g4_decoder_create_batch, one GPU, sliding-geometry layers): `batch` sequences per
    step; every layer's k_cache / v_cache is [batch, ring, Ns, Ds] (a ring per sequence), and
    input / hidden / logits hold one row per sequence."""

    def __init__(self, device: Device, layers: list[Layer], *, cos_local, sin_local, cos_global=None,
                 sin_global=None, embedding_table=None, final_norm_weight=None, lm_head_weight=None, cos_full=None,
                 sin_full=None, batch: int = 1):
        self.device = device
        self.batch = int(batch)
        self._keep = (layers, cos_local, sin_local, cos_global, sin_global, embedding_table, final_norm_weight,
                      lm_head_weight, cos_full, sin_full)
        arr = (_Layer * max(1, len(layers)))()
        for i, lay in enumerate(layers):
            s = arr[i]
            s.kind, s.rope, s.ring_len, s.ffn, s.tiled, s.attn_scale = lay.kind, lay.rope, lay.ring_len, lay.ffn, \
                int(lay.tiled), lay.attn_scale
            for f in fields(Layer):
                if f.name in ("kind", "rope", "ffn", "tiled", "attn_scale"):
                    continue
                setattr(s, f.name, _ptr(getattr(lay, f.name)).value)
        self._layers = arr
        m = _Model()
        m.layers = ctypes.cast(arr, ctypes.POINTER(_Layer))
        m.n_layers = len(layers)
        m.embedding_table = _ptr(embedding_table).value
        m.vocab_rows = embedding_table.shape[0] if embedding_table is not None else 0
        m.final_norm_weight = _ptr(final_norm_weight).value
        m.lm_head_weight = _ptr(lm_head_weight).value
        m.lm_head_rows = lm_head_weight.shape[0] if lm_head_weight is not None else 0
        m.cos_local, m.sin_local = _ptr(cos_local).value, _ptr(sin_local).value
        m.cos_global, m.sin_global = _ptr(cos_global).value, _ptr(sin_global).value
        m.rope_rows = cos_local.shape[0]
        m.cos_full, m.sin_full = _ptr(cos_full).value, _ptr(sin_full).value
        self._model = m
        self._dec = ctypes.c_void_p()
        _check(device, _abi.lib().g4_decoder_create_batch(device.handle, ctypes.byref(m), self.batch,
                                                          ctypes.byref(self._dec)), "g4_decoder_create_batch")
        inp, hid, log = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        _check(device, _abi.lib().g4_decoder_buffers(self._dec, ctypes.byref(inp), ctypes.byref(hid),
                                                      ctypes.byref(log)), "g4_decoder_buffers")
        self.input_ptr, self.hidden_ptr, self.logits_ptr = inp.value, hid.value, log.value
        self.lm_head_rows = m.lm_head_rows
        self._host_input = torch.zeros(2 * self.batch, dtype=torch.int32).pin_memory()

    def close(self) -> None:
        if self._dec:
            _abi.lib().g4_decoder_destroy(self._dec)
            self._dec = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def input_view(self) -> torch.Tensor:
        """The device-resident {token, position} (i32 [2], or [batch * 2]) as a tensor view."""
        return _device_view(self.input_ptr, 2 * self.batch, torch.int32, self.device.index)

    def hidden(self) -> torch.Tensor:
        """The hidden state [H] bf16 ([batch, H] for a batch; a view of the decoder's buffer)."""
        t = _device_view(self.hidden_ptr, 3840 * self.batch, torch.bfloat16, self.device.index)
        return t.view(self.batch, 3840) if self.batch > 1 else t

    def logits(self) -> torch.Tensor:
        if not self.logits_ptr:
            raise ValueError("the model has no lm_head")
        t = _device_view(self.logits_ptr, self.lm_head_rows * self.batch, torch.bfloat16, self.device.index)
        return t.view(self.batch, self.lm_head_rows) if self.batch > 1 else t

    def set_input(self, token, position, stream=None) -> None:
        """Write {token, position} on the stream (from pinned host memory); for a batch, one token
        and one position per sequence (sequences of length batch)."""
        s = stream if stream is not None else torch.cuda.current_stream(self.device.index)
        s.synchronize()  # the pinned staging buffer may still feed the previous copy
        tokens = [token] if self.batch == 1 and not hasattr(token, "__len__") else list(token)
        positions = [position] if self.batch == 1 and not hasattr(position, "__len__") else list(position)
        if len(tokens) != self.batch or len(positions) != self.batch:
            raise ValueError(f"expected {self.batch} tokens and positions")
        for i, (t, p) in enumerate(zip(tokens, positions)):
            self._host_input[2 * i], self._host_input[2 * i + 1] = int(t), int(p)
        with torch.cuda.stream(s):
            self.input_view().copy_(self._host_input, non_blocking=True)

    def step(self, token=None, position=None, stream=None) -> None:
        if token is not None:
            self.set_input(token, position, stream)
        _check(self.device, _abi.lib().g4_decoder_step(self._dec, _stream_ptr(stream, self.device.index)),
               "g4_decoder_step")

    def capture(self, stream=None) -> None:
        """Record one step as a CUDA graph (on a side stream unless one is given)."""
        s = stream if stream is not None else torch.cuda.Stream(self.device.index)
        s.wait_stream(torch.cuda.current_stream(self.device.index))
        _check(self.device, _abi.lib().g4_decoder_capture(self._dec, ctypes.c_void_p(s.cuda_stream)),
               "g4_decoder_capture")
        torch.cuda.current_stream(self.device.index).wait_stream(s)


def _device_view(ptr: int, n: int, dtype, index: int) -> torch.Tensor:
    """A tensor over n elements of device memory the library owns (no copy, not freed by torch)."""
    class _Holder:
        __cuda_array_interface__ = {"shape": (n,), "typestr": {torch.int32: "<i4", torch.bfloat16: "<i2"}[dtype],
                                    "data": (ptr, False), "version": 3, "strides": None}

    t = torch.as_tensor(_Holder(), device=f"cuda:{index}")
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t
