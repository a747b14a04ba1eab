"""Host mirror of the reference's device entry points (furiosa-opt-gemma4-12B/src/ops.rs).

Each function has the reference op's name and parameter order, takes CUDA tensors where the
reference takes `&HbmTensor` / `&mut HbmTensor`, checks the dtype and shape the reference
encodes in its types (`m![...]`, src/axes.rs:1-28) and calls the C ABI of libg4b200.so.
torch is only the device-memory and stream plumbing here; the computation is the library's.

Tensor encodings: bf16 -> torch.bfloat16; f8e4m3 -> torch.uint8 or torch.float8_e4m3fn;
packed f4e2m1 -> torch.uint8 [rows, cols/2]; f32 -> torch.float32; i32 -> torch.int32.
"""

from __future__ import annotations

import ctypes

import torch

from . import _abi
from ._abi import G4Error

H, L, NS, GS, DS, QS, PS, TS, E = 3840, 15360, 8, 2, 256, 4096, 2048, 1024, 32768


def geometry(world: int = 1) -> dict:
    """Per-rank sizes of a tensor-parallel split over `world` ranks (1 = the whole layer):
    KV heads, q rows, k/v rows, FFN rows (up/gate rows = down K) and the down K slice padded to
    whole 256-element units (include/g4b200.h, tensor parallelism)."""
    if world not in (1, 2, 4, 8):
        raise ValueError(f"tensor-parallel world must be 1, 2, 4 or 8, got {world}")
    ffn = L // world
    return {"kv_heads": NS // world, "q_rows": QS // world, "kv_rows": PS // world, "ffn_rows": ffn,
            "down_k": -(-ffn // 256) * 256}


class Device:
    """One GPU and its g4 context (the role of furiosa_opt_std's `Device`)."""

    def __init__(self, index: int = 0):
        self.index = index
        self.rank, self.world = 0, 1
        self._ctx = ctypes.c_void_p()
        st = _abi.lib().g4_ctx_create(index, ctypes.byref(self._ctx))
        if st != _abi.G4_OK:
            raise G4Error(st, f"g4_ctx_create(device={index}) failed")

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._ctx:
            raise RuntimeError("device context already closed")
        return self._ctx

    def close(self) -> None:
        if self._ctx:
            _abi.lib().g4_ctx_destroy(self._ctx)
            self._ctx = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_overlap(self, enable: bool) -> None:
        _check(self, _abi.lib().g4_ctx_set_overlap(self.handle, int(enable)), "g4_ctx_set_overlap")

    def check(self, stream: torch.cuda.Stream | None = None) -> None:
        """Synchronise the stream and raise if a kernel flagged a device-side error."""
        flags = ctypes.c_uint32(0)
        st = _abi.lib().g4_ctx_check(self.handle, _stream_ptr(stream, self.index), ctypes.byref(flags))
        if st != _abi.G4_OK:
            raise G4Error(st, f"device-side error flags 0x{flags.value:x}: {self.last_error()}", flags.value)

    def last_error(self) -> str:
        return _abi.lib().g4_last_error(self.handle).decode()

    def tp_init(self, rank: int, world: int) -> bytes:
        """g4_tp_init: make this context rank `rank` of a tensor-parallel group of `world` GPUs;
        returns the setup blob every other rank needs (see `g4b200.tp.connect`)."""
        blob = ctypes.create_string_buffer(_abi.TP_BLOB_BYTES)
        _check(self, _abi.lib().g4_tp_init(self.handle, rank, world, blob), "g4_tp_init")
        self.rank, self.world = rank, world
        return blob.raw

    def tp_set_wait_limit(self, seconds: float) -> None:
        """g4_tp_set_wait_limit: how long O / down wait for the peers before raising a peer timeout."""
        _check(self, _abi.lib().g4_tp_set_wait_limit(self.handle, int(seconds * 1e9)), "g4_tp_set_wait_limit")

    def tp_connect(self, blobs: bytes) -> None:
        """g4_tp_connect with every rank's blob, concatenated in rank order."""
        if len(blobs) != _abi.TP_BLOB_BYTES * self.world:
            raise ValueError(f"tp_connect: expected {self.world} blobs of {_abi.TP_BLOB_BYTES} bytes")
        buf = ctypes.create_string_buffer(blobs, len(blobs))
        _check(self, _abi.lib().g4_tp_connect(self.handle, buf), "g4_tp_connect")


def _stream_ptr(stream, device_index: int) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream(device_index)
    return ctypes.c_void_p(s.cuda_stream)


def _check(device: Device, status: int, what: str) -> None:
    if status != _abi.G4_OK:
        raise G4Error(status, f"{what}: {device.last_error()}")


_BYTE_DTYPES = (torch.uint8, torch.float8_e4m3fn)


def _arg(t: torch.Tensor, name: str, dtypes, shape, device: Device) -> ctypes.c_void_p:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name}: expected a torch.Tensor, got {type(t).__name__}")
    if t.dtype not in (dtypes if isinstance(dtypes, tuple) else (dtypes,)):
        raise TypeError(f"{name}: dtype {t.dtype}, expected {dtypes}")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {tuple(shape)}")
    if not t.is_cuda or t.device.index != device.index:
        raise ValueError(f"{name}: must live on cuda:{device.index}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: must be contiguous")
    return ctypes.c_void_p(t.data_ptr())


W = 262144  # vocabulary rows of the embedding / lm_head table


def embed_token(device: Device, embedding_table, offset, out, *, stream=None) -> None:
    """ops::embed_token (src/ops.rs:8-35): out = bf16(embedding_table[row] * 61.967734), the row at
    the device-resident BYTE offset `offset` (i32 [1], token * H * 2). embedding_table [rows, H]."""
    bf = torch.bfloat16
    rows = embedding_table.shape[0] if embedding_table.dim() == 2 else -1
    args = [_arg(embedding_table, "embedding_table", bf, (rows, H), device),
            _arg(offset, "offset", torch.int32, (1,), device), _arg(out, "out", bf, (H,), device)]
    st = _abi.lib().g4_embed_token(device.handle, *args, rows, _stream_ptr(stream, device.index))
    _check(device, st, "embed_token")


def final_norm_and_logits(device: Device, input, rms_weight, lm_head_weight, out, *, stream=None) -> None:
    """ops::final_norm_and_logits (src/ops.rs:241-298): out = softcap_30(bf16(RMSNorm(input) @
    lm_head_weight.T)). lm_head_weight [rows, H] (a tensor-parallel rank's slice of the W rows), out [rows]."""
    bf = torch.bfloat16
    rows = lm_head_weight.shape[0] if lm_head_weight.dim() == 2 else -1
    args = [_arg(input, "input", bf, (H,), device), _arg(rms_weight, "rms_weight", bf, (H,), device),
            _arg(lm_head_weight, "lm_head_weight", bf, (rows, H), device), _arg(out, "out", bf, (rows,), device)]
    st = _abi.lib().g4_final_norm_and_logits(device.handle, *args, rows, _stream_ptr(stream, device.index))
    _check(device, st, "final_norm_and_logits")


def final_norm_and_logits_batch(device: Device, input, rms_weight, lm_head_weight, out, *, stream=None) -> None:
    """final_norm_and_logits on each row of input [m, H] (m in [1, 64]), out [m, rows]: the table is
    read once for all m (tcgen05 tiles when rows is a multiple of 128)."""
    bf = torch.bfloat16
    m = _batch_of(input, "input", 2)
    rows = lm_head_weight.shape[0] if lm_head_weight.dim() == 2 else -1
    args = [_arg(input, "input", bf, (m, H), device), _arg(rms_weight, "rms_weight", bf, (H,), device),
            _arg(lm_head_weight, "lm_head_weight", bf, (rows, H), device), _arg(out, "out", bf, (m, rows), device)]
    st = _abi.lib().g4_final_norm_and_logits_batch(device.handle, *args, rows, m, _stream_ptr(stream, device.index))
    _check(device, st, "final_norm_and_logits_batch")


GF, DF, QF, TF = 16, 512, 8192, 512  # global layers: query heads, head dim, q rows, page slots


def full_project_qkv(device: Device, x, q_weight, k_weight, q_weight_scale, k_weight_scale, input_rms_weight,
                     q_rms_weight, k_rms_weight, kv_offset, rope_offset, cos, sin, k_cache, v_cache, q_out, *,
                     stream=None) -> None:
    """ops::full_project_qkv (src/ops.rs:78-116). k_cache / v_cache: the current page [Tf, Df];
    cos / sin: [rows, Df] (the global table). One GPU only."""
    bf = torch.bfloat16
    rows = cos.shape[0] if cos.dim() == 2 else -1
    args = [
        _arg(x, "x", bf, (H,), device),
        _arg(q_weight, "q_weight", _BYTE_DTYPES, (QF, H), device),
        _arg(k_weight, "k_weight", _BYTE_DTYPES, (DF, H), device),
        _arg(q_weight_scale, "q_weight_scale", bf, (QF,), device),
        _arg(k_weight_scale, "k_weight_scale", bf, (DF,), device),
        _arg(input_rms_weight, "input_rms_weight", bf, (H,), device),
        _arg(q_rms_weight, "q_rms_weight", bf, (DF,), device),
        _arg(k_rms_weight, "k_rms_weight", bf, (DF,), device),
        _arg(kv_offset, "kv_offset", torch.int32, (1,), device),
        _arg(rope_offset, "rope_offset", torch.int32, (1,), device),
        _arg(cos, "cos", bf, (rows, DF), device),
        _arg(sin, "sin", bf, (rows, DF), device),
        _arg(k_cache, "k_cache", bf, (TF, DF), device),
        _arg(v_cache, "v_cache", bf, (TF, DF), device),
        _arg(q_out, "q_out", bf, (GF, DF), device),
    ]
    st = _abi.lib().g4_full_project_qkv(device.handle, *args, rows, _stream_ptr(stream, device.index))
    _check(device, st, "full_project_qkv")


def full_attention_page(device: Device, q, k, v, mask, running_max, running_sum, out_hbm, *, first: bool,
                        stream=None) -> None:
    """ops::full_attention_first_page (first=True) / ops::full_attention_page (src/ops.rs:148-182):
    one page [Tf, Df] of K and V; running_max / running_sum [Gf] f32 and out_hbm [Gf, Df] carry the
    online softmax from page to page."""
    bf = torch.bfloat16
    args = [_arg(q, "q", bf, (GF, DF), device), _arg(k, "k", bf, (TF, DF), device),
            _arg(v, "v", bf, (TF, DF), device), _arg(mask, "mask", torch.float32, (TF,), device),
            _arg(running_max, "running_max", torch.float32, (GF,), device),
            _arg(running_sum, "running_sum", torch.float32, (GF,), device),
            _arg(out_hbm, "out_hbm", bf, (GF, DF), device)]
    fn = _abi.lib().g4_full_attention_first_page if first else _abi.lib().g4_full_attention_page
    _check(device, fn(device.handle, *args, _stream_ptr(stream, device.index)), "full_attention_page")


def full_attention_output(device: Device, x, running_sum, post_attn_rms_weight, o_weight, o_weight_scale,
                          residual_hbm, *, stream=None) -> None:
    """ops::full_attention_output (src/ops.rs:184-199). residual_hbm is updated in place."""
    bf = torch.bfloat16
    args = [_arg(x, "x", bf, (GF, DF), device), _arg(running_sum, "running_sum", torch.float32, (GF,), device),
            _arg(post_attn_rms_weight, "post_attn_rms_weight", bf, (H,), device),
            _arg(o_weight, "o_weight", _BYTE_DTYPES, (H, QF), device),
            _arg(o_weight_scale, "o_weight_scale", bf, (H,), device),
            _arg(residual_hbm, "residual_hbm", bf, (H,), device)]
    st = _abi.lib().g4_full_attention_output(device.handle, *args, _stream_ptr(stream, device.index))
    _check(device, st, "full_attention_output")


def sliding_project_qkv(device: Device, x, q_weight, k_weight, v_weight, q_weight_scale, k_weight_scale,
                        v_weight_scale, input_rms_weight, q_rms_weight, k_rms_weight, kv_offset, rope_offset,
                        cos, sin, k_cache, v_cache, q_out, *, tiled=False, stream=None) -> None:
    """ops::sliding_project_qkv (src/ops.rs:37-76). k_cache/v_cache: [ring, Ns, Ds]; cos/sin: [rows, Ds].

    tiled=True: q/k/v weights are in the unit-tiled layout made by `pack_tiles` (TILING).
    On a tensor-parallel device the weights, caches and q_out are this rank's slices (`geometry`)."""
    bf = torch.bfloat16
    g = geometry(device.world)
    qr, kr, nh = g["q_rows"], g["kv_rows"], g["kv_heads"]
    ring = k_cache.shape[0] if k_cache.dim() == 3 else -1
    rows = cos.shape[0] if cos.dim() == 2 else -1
    args = [
        _arg(x, "x", bf, (H,), device),
        _arg(q_weight, "q_weight", _BYTE_DTYPES, (qr, H), device),
        _arg(k_weight, "k_weight", _BYTE_DTYPES, (kr, H), device),
        _arg(v_weight, "v_weight", _BYTE_DTYPES, (kr, H), device),
        _arg(q_weight_scale, "q_weight_scale", bf, (qr,), device),
        _arg(k_weight_scale, "k_weight_scale", bf, (kr,), device),
        _arg(v_weight_scale, "v_weight_scale", bf, (kr,), device),
        _arg(input_rms_weight, "input_rms_weight", bf, (H,), device),
        _arg(q_rms_weight, "q_rms_weight", bf, (DS,), device),
        _arg(k_rms_weight, "k_rms_weight", bf, (DS,), device),
        _arg(kv_offset, "kv_offset", torch.int32, (1,), device),
        _arg(rope_offset, "rope_offset", torch.int32, (1,), device),
        _arg(cos, "cos", bf, (rows, DS), device),
        _arg(sin, "sin", bf, (rows, DS), device),
        _arg(k_cache, "k_cache", bf, (ring, nh, DS), device),
        _arg(v_cache, "v_cache", bf, (ring, nh, DS), device),
        _arg(q_out, "q_out", bf, (nh, GS, DS), device),
    ]
    fn = _abi.lib().g4_sliding_project_qkv_tiled if tiled else _abi.lib().g4_sliding_project_qkv
    st = fn(device.handle, *args, ring, rows, _stream_ptr(stream, device.index))
    _check(device, st, "sliding_project_qkv")


def sliding_attention(device: Device, q, k, v, mask, out_hbm, *, scale: float = 1.0, kv_offset=None,
                      stream=None) -> None:
    """ops::sliding_attention (src/ops.rs:118-128). k/v: [ring, Ns, Ds]; mask: [ring] f32.

    On a tensor-parallel device q, k, v and out_hbm are this rank's heads (`geometry`).
    kv_offset: the i32 [1] the layer's sliding_project_qkv just got on the same stream; the
    kernel then copies every other cache row while that op finishes (g4_sliding_attention_after_qkv)."""
    bf = torch.bfloat16
    nh = geometry(device.world)["kv_heads"]
    ring = k.shape[0] if k.dim() == 3 else -1
    args = [
        _arg(q, "q", bf, (nh, GS, DS), device),
        _arg(k, "k", bf, (ring, nh, DS), device),
        _arg(v, "v", bf, (ring, nh, DS), device),
        _arg(mask, "mask", torch.float32, (ring,), device),
        _arg(out_hbm, "out_hbm", bf, (nh, GS, DS), device),
    ]
    if kv_offset is None:
        st = _abi.lib().g4_sliding_attention(device.handle, *args, ring, float(scale), _stream_ptr(stream, device.index))
    else:
        st = _abi.lib().g4_sliding_attention_after_qkv(device.handle, *args, ring, float(scale),
                                                       _arg(kv_offset, "kv_offset", torch.int32, (1,), device),
                                                       _stream_ptr(stream, device.index))
    _check(device, st, "sliding_attention")


def sliding_attention_output(device: Device, x, post_attn_rms_weight, o_weight, o_weight_scale, residual_hbm, *,
                             tiled=False, stream=None) -> None:
    """ops::sliding_attention_output (src/ops.rs:130-146). residual_hbm is updated in place.

    tiled=True: o_weight is in the unit-tiled layout made by `pack_tiles` (TILING).
    On a tensor-parallel device x is this rank's attention output and o_weight its K columns."""
    bf = torch.bfloat16
    g = geometry(device.world)
    args = [
        _arg(x, "x", bf, (g["kv_heads"], GS, DS), device),
        _arg(post_attn_rms_weight, "post_attn_rms_weight", bf, (H,), device),
        _arg(o_weight, "o_weight", _BYTE_DTYPES, (H, g["q_rows"]), device),
        _arg(o_weight_scale, "o_weight_scale", bf, (H,), device),
        _arg(residual_hbm, "residual_hbm", bf, (H,), device),
    ]
    fn = _abi.lib().g4_sliding_attention_output_tiled if tiled else _abi.lib().g4_sliding_attention_output
    st = fn(device.handle, *args, _stream_ptr(stream, device.index))
    _check(device, st, "sliding_attention_output")


def decoder_feedforward(device: Device, residual_hbm, pre_ff_rms_weight, up_weight_packed, gate_weight_packed,
                        down_weight_packed, up_weight_scale, gate_weight_scale, down_weight_scale, up_global_scale,
                        gate_global_scale, down_global_scale, post_ff_rms_weight, layer_scalar, *,
                        stream=None) -> None:
    """ops::decoder_feedforward (src/ops.rs:201-239). residual_hbm is updated in place.

    *_global_scale hold the reciprocal of the checkpoint's global scale (src/host/load.rs:170-190).
    On a tensor-parallel device the up/gate rows and down columns are this rank's slices.
    """
    bf = torch.bfloat16
    g = geometry(device.world)
    fr, dk = g["ffn_rows"], g["down_k"]
    args = [
        _arg(residual_hbm, "residual_hbm", bf, (H,), device),
        _arg(pre_ff_rms_weight, "pre_ff_rms_weight", bf, (H,), device),
        _arg(up_weight_packed, "up_weight_packed", torch.uint8, (fr, H // 2), device),
        _arg(gate_weight_packed, "gate_weight_packed", torch.uint8, (fr, H // 2), device),
        _arg(down_weight_packed, "down_weight_packed", torch.uint8, (H, dk // 2), device),
        _arg(up_weight_scale, "up_weight_scale", _BYTE_DTYPES, (fr, H // 16), device),
        _arg(gate_weight_scale, "gate_weight_scale", _BYTE_DTYPES, (fr, H // 16), device),
        _arg(down_weight_scale, "down_weight_scale", _BYTE_DTYPES, (H, dk // 16), device),
        _arg(up_global_scale, "up_global_scale", torch.float32, (1,), device),
        _arg(gate_global_scale, "gate_global_scale", torch.float32, (1,), device),
        _arg(down_global_scale, "down_global_scale", torch.float32, (1,), device),
        _arg(post_ff_rms_weight, "post_ff_rms_weight", bf, (H,), device),
        _arg(layer_scalar, "layer_scalar", bf, (8,), device),
    ]
    st = _abi.lib().g4_decoder_feedforward(device.handle, *args, _stream_ptr(stream, device.index))
    _check(device, st, "decoder_feedforward")


def decoder_feedforward_tiled(device: Device, residual_hbm, pre_ff_rms_weight, up_gate_weight_tiled,
                              down_weight_tiled, up_gate_scale_tiled, down_scale_tiled, up_global_scale,
                              gate_global_scale, down_global_scale, post_ff_rms_weight, layer_scalar, *,
                              stream=None) -> None:
    """decoder_feedforward on weights packed by `pack_upgate` / `tile_weight` (the GPU-native layout)."""
    bf = torch.bfloat16
    g = geometry(device.world)
    fr, dk = g["ffn_rows"], g["down_k"]
    args = [
        _arg(residual_hbm, "residual_hbm", bf, (H,), device),
        _arg(pre_ff_rms_weight, "pre_ff_rms_weight", bf, (H,), device),
        _arg(up_gate_weight_tiled, "up_gate_weight_tiled", torch.uint8, (2 * fr, H // 2), device),
        _arg(down_weight_tiled, "down_weight_tiled", torch.uint8, (H, dk // 2), device),
        _arg(up_gate_scale_tiled, "up_gate_scale_tiled", _BYTE_DTYPES, (2 * fr, H // 16), device),
        _arg(down_scale_tiled, "down_scale_tiled", _BYTE_DTYPES, (H, dk // 16), device),
        _arg(up_global_scale, "up_global_scale", torch.float32, (1,), device),
        _arg(gate_global_scale, "gate_global_scale", torch.float32, (1,), device),
        _arg(down_global_scale, "down_global_scale", torch.float32, (1,), device),
        _arg(post_ff_rms_weight, "post_ff_rms_weight", bf, (H,), device),
        _arg(layer_scalar, "layer_scalar", bf, (8,), device),
    ]
    st = _abi.lib().g4_decoder_feedforward_tiled(device.handle, *args, _stream_ptr(stream, device.index))
    _check(device, st, "decoder_feedforward_tiled")


BATCH_MAX = 64  # tokens per decoder_feedforward_batch call


def _batch_rows(residual_hbm) -> int:
    m = residual_hbm.shape[0] if residual_hbm.dim() == 2 else 0
    if not 1 <= m <= BATCH_MAX:
        raise ValueError(f"residual_hbm: shape {tuple(residual_hbm.shape)}, expected [m, {H}] with m in [1, {BATCH_MAX}]")
    return m


def decoder_feedforward_batch(device: Device, residual_hbm, pre_ff_rms_weight, up_weight_packed, gate_weight_packed,
                              down_weight_packed, up_weight_scale, gate_weight_scale, down_weight_scale,
                              up_global_scale, gate_global_scale, down_global_scale, post_ff_rms_weight, layer_scalar,
                              *, stream=None) -> None:
    """decoder_feedforward (src/ops.rs:201-239) on each row of residual_hbm [m, H], m in [1, 64]:
    the weights are read once for all m tokens (the NVFP4 token-batch sweep). One GPU."""
    bf = torch.bfloat16
    m = _batch_rows(residual_hbm)
    args = [
        _arg(residual_hbm, "residual_hbm", bf, (m, H), device),
        _arg(pre_ff_rms_weight, "pre_ff_rms_weight", bf, (H,), device),
        _arg(up_weight_packed, "up_weight_packed", torch.uint8, (L, H // 2), device),
        _arg(gate_weight_packed, "gate_weight_packed", torch.uint8, (L, H // 2), device),
        _arg(down_weight_packed, "down_weight_packed", torch.uint8, (H, L // 2), device),
        _arg(up_weight_scale, "up_weight_scale", _BYTE_DTYPES, (L, H // 16), device),
        _arg(gate_weight_scale, "gate_weight_scale", _BYTE_DTYPES, (L, H // 16), device),
        _arg(down_weight_scale, "down_weight_scale", _BYTE_DTYPES, (H, L // 16), device),
        _arg(up_global_scale, "up_global_scale", torch.float32, (1,), device),
        _arg(gate_global_scale, "gate_global_scale", torch.float32, (1,), device),
        _arg(down_global_scale, "down_global_scale", torch.float32, (1,), device),
        _arg(post_ff_rms_weight, "post_ff_rms_weight", bf, (H,), device),
        _arg(layer_scalar, "layer_scalar", bf, (8,), device),
    ]
    st = _abi.lib().g4_decoder_feedforward_batch(device.handle, *args, m, _stream_ptr(stream, device.index))
    _check(device, st, "decoder_feedforward_batch")


def decoder_feedforward_batch_tiled(device: Device, residual_hbm, pre_ff_rms_weight, up_gate_weight_tiled,
                                    down_weight_tiled, up_gate_scale_tiled, down_scale_tiled, up_global_scale,
                                    gate_global_scale, down_global_scale, post_ff_rms_weight, layer_scalar, *,
                                    stream=None) -> None:
    """decoder_feedforward_batch on weights packed by `pack_upgate` / `tile_weight`."""
    bf = torch.bfloat16
    m = _batch_rows(residual_hbm)
    args = [
        _arg(residual_hbm, "residual_hbm", bf, (m, H), device),
        _arg(pre_ff_rms_weight, "pre_ff_rms_weight", bf, (H,), device),
        _arg(up_gate_weight_tiled, "up_gate_weight_tiled", torch.uint8, (2 * L, H // 2), device),
        _arg(down_weight_tiled, "down_weight_tiled", torch.uint8, (H, L // 2), device),
        _arg(up_gate_scale_tiled, "up_gate_scale_tiled", _BYTE_DTYPES, (2 * L, H // 16), device),
        _arg(down_scale_tiled, "down_scale_tiled", _BYTE_DTYPES, (H, L // 16), device),
        _arg(up_global_scale, "up_global_scale", torch.float32, (1,), device),
        _arg(gate_global_scale, "gate_global_scale", torch.float32, (1,), device),
        _arg(down_global_scale, "down_global_scale", torch.float32, (1,), device),
        _arg(post_ff_rms_weight, "post_ff_rms_weight", bf, (H,), device),
        _arg(layer_scalar, "layer_scalar", bf, (8,), device),
    ]
    st = _abi.lib().g4_decoder_feedforward_batch_tiled(device.handle, *args, m, _stream_ptr(stream, device.index))
    _check(device, st, "decoder_feedforward_batch_tiled")


def decoder_feedforward_fp8(device: Device, residual_hbm, pre_ff_rms_weight, up_weight, gate_weight, down_weight,
                            up_weight_scale, gate_weight_scale, down_weight_scale, post_ff_rms_weight, layer_scalar, *,
                            stream=None) -> None:
    """The GeGLU feed-forward on FP8 weights with f32 per-output-channel scales (BASELINE
    configs[0]): decoder_feedforward's epilogue (src/ops.rs:201-239) around three scaled
    projections (scripts/generate_references.py:265-274). residual_hbm is updated in place.

    up/gate_weight [L, H] and down_weight [H, L] e4m3; up/gate_weight_scale [L] and
    down_weight_scale [H] f32. On a tensor-parallel device the up/gate rows (and their scales)
    and the down columns are this rank's slices (g4b200.tp names: up_weight, gate_weight,
    down_weight, up_channel_scale, gate_channel_scale, down_channel_scale)."""
    bf = torch.bfloat16
    g = geometry(device.world)
    fr, dk = g["ffn_rows"], g["down_k"]
    args = [
        _arg(residual_hbm, "residual_hbm", bf, (H,), device),
        _arg(pre_ff_rms_weight, "pre_ff_rms_weight", bf, (H,), device),
        _arg(up_weight, "up_weight", _BYTE_DTYPES, (fr, H), device),
        _arg(gate_weight, "gate_weight", _BYTE_DTYPES, (fr, H), device),
        _arg(down_weight, "down_weight", _BYTE_DTYPES, (H, dk), device),
        _arg(up_weight_scale, "up_weight_scale", torch.float32, (fr,), device),
        _arg(gate_weight_scale, "gate_weight_scale", torch.float32, (fr,), device),
        _arg(down_weight_scale, "down_weight_scale", torch.float32, (H,), device),
        _arg(post_ff_rms_weight, "post_ff_rms_weight", bf, (H,), device),
        _arg(layer_scalar, "layer_scalar", bf, (8,), device),
    ]
    st = _abi.lib().g4_decoder_feedforward_fp8(device.handle, *args, _stream_ptr(stream, device.index))
    _check(device, st, "decoder_feedforward_fp8")


def decoder_feedforward_fp8_tiled(device: Device, residual_hbm, pre_ff_rms_weight, up_gate_weight_tiled,
                                  down_weight_tiled, up_weight_scale, gate_weight_scale, down_weight_scale,
                                  post_ff_rms_weight, layer_scalar, *, stream=None) -> None:
    """decoder_feedforward_fp8 on weights packed by `pack_upgate_fp8` / `tile_weight(.., "down_weight")`."""
    bf = torch.bfloat16
    g = geometry(device.world)
    fr, dk = g["ffn_rows"], g["down_k"]
    args = [
        _arg(residual_hbm, "residual_hbm", bf, (H,), device),
        _arg(pre_ff_rms_weight, "pre_ff_rms_weight", bf, (H,), device),
        _arg(up_gate_weight_tiled, "up_gate_weight_tiled", _BYTE_DTYPES, (2 * fr, H), device),
        _arg(down_weight_tiled, "down_weight_tiled", _BYTE_DTYPES, (H, dk), device),
        _arg(up_weight_scale, "up_weight_scale", torch.float32, (fr,), device),
        _arg(gate_weight_scale, "gate_weight_scale", torch.float32, (fr,), device),
        _arg(down_weight_scale, "down_weight_scale", torch.float32, (H,), device),
        _arg(post_ff_rms_weight, "post_ff_rms_weight", bf, (H,), device),
        _arg(layer_scalar, "layer_scalar", bf, (8,), device),
    ]
    st = _abi.lib().g4_decoder_feedforward_fp8_tiled(device.handle, *args, _stream_ptr(stream, device.index))
    _check(device, st, "decoder_feedforward_fp8_tiled")


def _batch_of(t, name, dims) -> int:
    m = t.shape[0] if t.dim() == dims else 0
    if not 1 <= m <= BATCH_MAX:
        raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {dims} dimensions with the first, m, in [1, {BATCH_MAX}]")
    return m


def sliding_project_qkv_batch(device: Device, x, q_weight, k_weight, v_weight, q_weight_scale, k_weight_scale,
                              v_weight_scale, input_rms_weight, q_rms_weight, k_rms_weight, kv_offset, rope_offset,
                              cos, sin, k_cache, v_cache, q_out, *, tiled=False, stream=None) -> None:
    """sliding_project_qkv (src/ops.rs:37-76) on each of m sequences, the weights read once for all m:
    x [m, H]; kv_offset / rope_offset [m] i32 byte offsets; k_cache / v_cache [m, ring, Ns, Ds]
    (sequence i's ring at [i]); q_out [m, Ns, Gs, Ds]. m in [1, 64]; one GPU."""
    bf = torch.bfloat16
    m = _batch_of(x, "x", 2)
    ring = k_cache.shape[1] if k_cache.dim() == 4 else -1
    rows = cos.shape[0] if cos.dim() == 2 else -1
    args = [
        _arg(x, "x", bf, (m, H), device),
        _arg(q_weight, "q_weight", _BYTE_DTYPES, (QS, H), device),
        _arg(k_weight, "k_weight", _BYTE_DTYPES, (PS, H), device),
        _arg(v_weight, "v_weight", _BYTE_DTYPES, (PS, H), device),
        _arg(q_weight_scale, "q_weight_scale", bf, (QS,), device),
        _arg(k_weight_scale, "k_weight_scale", bf, (PS,), device),
        _arg(v_weight_scale, "v_weight_scale", bf, (PS,), device),
        _arg(input_rms_weight, "input_rms_weight", bf, (H,), device),
        _arg(q_rms_weight, "q_rms_weight", bf, (DS,), device),
        _arg(k_rms_weight, "k_rms_weight", bf, (DS,), device),
        _arg(kv_offset, "kv_offset", torch.int32, (m,), device),
        _arg(rope_offset, "rope_offset", torch.int32, (m,), device),
        _arg(cos, "cos", bf, (rows, DS), device),
        _arg(sin, "sin", bf, (rows, DS), device),
        _arg(k_cache, "k_cache", bf, (m, ring, NS, DS), device),
        _arg(v_cache, "v_cache", bf, (m, ring, NS, DS), device),
        _arg(q_out, "q_out", bf, (m, NS, GS, DS), device),
    ]
    fn = _abi.lib().g4_sliding_project_qkv_batch_tiled if tiled else _abi.lib().g4_sliding_project_qkv_batch
    st = fn(device.handle, *args, ring, rows, m, _stream_ptr(stream, device.index))
    _check(device, st, "sliding_project_qkv_batch")


def sliding_attention_batch(device: Device, q, k, v, mask, out_hbm, *, scale: float = 1.0, kv_offset=None,
                            stream=None) -> None:
    """sliding_attention (src/ops.rs:118-128) on each of m sequences: q / out_hbm [m, Ns, Gs, Ds],
    k / v [m, ring, Ns, Ds], mask [m, ring] f32, kv_offset None or the [m] i32 the batched QKV op
    just got. m in [1, 64]; one GPU."""
    bf = torch.bfloat16
    m = _batch_of(q, "q", 4)
    ring = k.shape[1] if k.dim() == 4 else -1
    args = [
        _arg(q, "q", bf, (m, NS, GS, DS), device),
        _arg(k, "k", bf, (m, ring, NS, DS), device),
        _arg(v, "v", bf, (m, ring, NS, DS), device),
        _arg(mask, "mask", torch.float32, (m, ring), device),
        _arg(out_hbm, "out_hbm", bf, (m, NS, GS, DS), device),
    ]
    off = None if kv_offset is None else _arg(kv_offset, "kv_offset", torch.int32, (m,), device)
    st = _abi.lib().g4_sliding_attention_batch(device.handle, *args, ring, float(scale), off, m,
                                               _stream_ptr(stream, device.index))
    _check(device, st, "sliding_attention_batch")


def sliding_attention_output_batch(device: Device, x, post_attn_rms_weight, o_weight, o_weight_scale, residual_hbm, *,
                                   tiled=False, stream=None) -> None:
    """sliding_attention_output (src/ops.rs:130-146) on each of m sequences: x [m, Ns, Gs, Ds],
    residual_hbm [m, H] updated in place; the O weights read once for all m. m in [1, 64]; one GPU."""
    bf = torch.bfloat16
    m = _batch_of(residual_hbm, "residual_hbm", 2)
    args = [
        _arg(x, "x", bf, (m, NS, GS, DS), device),
        _arg(post_attn_rms_weight, "post_attn_rms_weight", bf, (H,), device),
        _arg(o_weight, "o_weight", _BYTE_DTYPES, (H, QS), device),
        _arg(o_weight_scale, "o_weight_scale", bf, (H,), device),
        _arg(residual_hbm, "residual_hbm", bf, (m, H), device),
    ]
    fn = (_abi.lib().g4_sliding_attention_output_batch_tiled if tiled
          else _abi.lib().g4_sliding_attention_output_batch)
    st = fn(device.handle, *args, m, _stream_ptr(stream, device.index))
    _check(device, st, "sliding_attention_output_batch")


def decoder_feedforward_fp8_batch(device: Device, residual_hbm, pre_ff_rms_weight, up_weight, gate_weight, down_weight,
                                  up_weight_scale, gate_weight_scale, down_weight_scale, post_ff_rms_weight,
                                  layer_scalar, *, stream=None) -> None:
    """decoder_feedforward_fp8 on each row of residual_hbm [m, H], m in [1, 64]: the weights are
    read once for all m tokens. One GPU."""
    bf = torch.bfloat16
    m = _batch_rows(residual_hbm)
    args = [
        _arg(residual_hbm, "residual_hbm", bf, (m, H), device),
        _arg(pre_ff_rms_weight, "pre_ff_rms_weight", bf, (H,), device),
        _arg(up_weight, "up_weight", _BYTE_DTYPES, (L, H), device),
        _arg(gate_weight, "gate_weight", _BYTE_DTYPES, (L, H), device),
        _arg(down_weight, "down_weight", _BYTE_DTYPES, (H, L), device),
        _arg(up_weight_scale, "up_weight_scale", torch.float32, (L,), device),
        _arg(gate_weight_scale, "gate_weight_scale", torch.float32, (L,), device),
        _arg(down_weight_scale, "down_weight_scale", torch.float32, (H,), device),
        _arg(post_ff_rms_weight, "post_ff_rms_weight", bf, (H,), device),
        _arg(layer_scalar, "layer_scalar", bf, (8,), device),
    ]
    st = _abi.lib().g4_decoder_feedforward_fp8_batch(device.handle, *args, m, _stream_ptr(stream, device.index))
    _check(device, st, "decoder_feedforward_fp8_batch")


def decoder_feedforward_fp8_batch_tiled(device: Device, residual_hbm, pre_ff_rms_weight, up_gate_weight_tiled,
                                        down_weight_tiled, up_weight_scale, gate_weight_scale, down_weight_scale,
                                        post_ff_rms_weight, layer_scalar, *, stream=None) -> None:
    """decoder_feedforward_fp8_batch on weights packed by `pack_upgate_fp8` / `tile_weight(.., "down_weight")`."""
    bf = torch.bfloat16
    m = _batch_rows(residual_hbm)
    args = [
        _arg(residual_hbm, "residual_hbm", bf, (m, H), device),
        _arg(pre_ff_rms_weight, "pre_ff_rms_weight", bf, (H,), device),
        _arg(up_gate_weight_tiled, "up_gate_weight_tiled", _BYTE_DTYPES, (2 * L, H), device),
        _arg(down_weight_tiled, "down_weight_tiled", _BYTE_DTYPES, (H, L), device),
        _arg(up_weight_scale, "up_weight_scale", torch.float32, (L,), device),
        _arg(gate_weight_scale, "gate_weight_scale", torch.float32, (L,), device),
        _arg(down_weight_scale, "down_weight_scale", torch.float32, (H,), device),
        _arg(post_ff_rms_weight, "post_ff_rms_weight", bf, (H,), device),
        _arg(layer_scalar, "layer_scalar", bf, (8,), device),
    ]
    st = _abi.lib().g4_decoder_feedforward_fp8_batch_tiled(device.handle, *args, m, _stream_ptr(stream, device.index))
    _check(device, st, "decoder_feedforward_fp8_batch_tiled")


# GPU-native (unit-tiled) layout of each weight matrix: (unit_bytes, tile_rows). A unit is the
# 256 K elements of a tile of rows (fp8: one tensor-memory-accelerator box of two 128-element
# halves; nvfp4: 128 bytes of packed codes, or 16 block-scale bytes, per row); the units of a
# tile are contiguous in memory. The up and gate matrices (codes and scales) are interleaved
# into one buffer each by `pack_upgate`.
TILING = {
    "q_weight": (128, 128), "k_weight": (128, 128), "v_weight": (128, 128), "o_weight": (128, 128),
    "up_gate_weight": (128, 64), "up_gate_scale": (16, 64),
    "down_weight_packed": (128, 128), "down_weight_scale": (16, 128),
    "up_gate_weight_fp8": (128, 64), "down_weight": (128, 128),
}


def pack_tiles(device: Device, src: torch.Tensor, src2: torch.Tensor | None = None, *, unit_bytes: int,
               tile_rows: int, stream=None) -> torch.Tensor:
    """src (and src2, interleaved tile by tile) [rows, row_bytes] in the unit-tiled layout; the
    result has shape [rows * n_sources, row_bytes]. The weights are static: pack them once at load."""
    if src.dim() != 2 or src.element_size() != 1:
        raise ValueError("pack_tiles: expects a 2-D byte matrix")
    if src2 is not None and (src2.shape != src.shape or src2.dtype != src.dtype):
        raise ValueError("pack_tiles: src2 must match src")
    n = 1 if src2 is None else 2
    dst = torch.empty((src.shape[0] * n, src.shape[1]), dtype=src.dtype, device=src.device)
    st = _abi.lib().g4_pack_tiles(device.handle, _arg(src, "src", src.dtype, None, device),
                                  None if src2 is None else _arg(src2, "src2", src2.dtype, None, device),
                                  _arg(dst, "dst", dst.dtype, None, device), src.shape[0], src.shape[1], unit_bytes,
                                  tile_rows, _stream_ptr(stream, device.index))
    _check(device, st, "pack_tiles")
    return dst


def tile_weight(device: Device, name: str, src: torch.Tensor, *, stream=None) -> torch.Tensor:
    """`src` (the reference layout of weight `name`: q/k/v/o_weight, down_weight_packed or
    down_weight_scale) in the GPU-native layout."""
    unit_bytes, tile_rows = TILING[name]
    return pack_tiles(device, src, unit_bytes=unit_bytes, tile_rows=tile_rows, stream=stream)


def pack_upgate(device: Device, up: torch.Tensor, gate: torch.Tensor, *, scales: bool, stream=None) -> torch.Tensor:
    """The up and gate packed codes (scales=False) or block scales (scales=True), interleaved in
    the GPU-native layout of decoder_feedforward_tiled."""
    unit_bytes, tile_rows = TILING["up_gate_scale" if scales else "up_gate_weight"]
    return pack_tiles(device, up, gate, unit_bytes=unit_bytes, tile_rows=tile_rows, stream=stream)


def pack_upgate_fp8(device: Device, up: torch.Tensor, gate: torch.Tensor, *, stream=None) -> torch.Tensor:
    """The FP8 up and gate codes interleaved in the GPU-native layout of decoder_feedforward_fp8_tiled."""
    unit_bytes, tile_rows = TILING["up_gate_weight_fp8"]
    return pack_tiles(device, up, gate, unit_bytes=unit_bytes, tile_rows=tile_rows, stream=stream)
