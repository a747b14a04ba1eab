"""Byte-exact input synthesis for the parity harness (TEST INFRASTRUCTURE, not product code).

This module is part of the CPU oracle. Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` may import it, and only as the
checker. The CUDA path never calls it.

It restates the reference harness's stateless PRNG so that the same (run, test, name)
triple yields the same bytes the reference fed its kernels:

- `name_hash`      FNV-1a over the UTF-8 name      FOG/scripts/fixture_prng.py:44-54
- `words`          splitmix64 finaliser over index FOG/scripts/fixture_prng.py:57-67
- `u01`            top 24 bits / 2**24             FOG/scripts/fixture_prng.py:71-77
- `f32_to_bf16_bits` round-half-to-even            FOG/scripts/fixture_prng.py:80-90
- `bf16_uniform`   lo + (hi-lo)*u in f32           FOG/scripts/fixture_prng.py:94-102
- `f32_uniform`                                     FOG/scripts/fixture_prng.py:105-112
- `bf16_signs`     +/-scale from the top bit       FOG/scripts/fixture_prng.py:115-125
- `f8_banded`      e4m3 codes from bit fields      FOG/scripts/fixture_prng.py:128-148
- `f4_nibbles`     e2m1 codes, low nibble first    FOG/scripts/fixture_prng.py:151-166
- `checksum`       position-weighted u32 sum       FOG/scripts/fixture_prng.py:170-198

(`FOG` = `furiosa-opt-gemma4-12B/` in the reference workspace.) The Rust mirror of the same
algorithm is FOG/src/bin/test_kernels.rs:34-145. The constants are the published
splitmix64 / FNV-1a constants; they must be identical for the bytes to agree.

Large tensors go through the C restatement in `oracle/c/g4oracle.c` when it has been built
(`oracle/_build/libg4oracle.so`), which produces identical bytes far faster; the numpy
path below is the definition and is used whenever the library is absent.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

MASK64 = 0xFFFF_FFFF_FFFF_FFFF
FNV_OFFSET = 0xCBF2_9CE4_8422_2325
FNV_PRIME = 0x0000_0100_0000_01B3
GOLDEN = np.uint64(0x9E37_79B9_7F4A_7C15)
MIX_A = np.uint64(0xBF58_476D_1CE4_E5B9)
MIX_B = np.uint64(0x94D0_49BB_1331_11EB)

_LIB = None
_LIB_PATH = Path(__file__).resolve().parent / "_build" / "libg4oracle.so"


def _lib():
    """The optional C restatement (same algorithm, OpenMP-parallel)."""
    global _LIB
    if _LIB is None:
        if _LIB_PATH.exists() and not os.environ.get("G4_ORACLE_NUMPY_ONLY"):
            lib = ctypes.CDLL(str(_LIB_PATH))
            u8p = ctypes.POINTER(ctypes.c_uint8)
            lib.g4o_f4_nibbles.argtypes = [ctypes.c_uint64, ctypes.c_size_t, u8p]
            lib.g4o_f8_banded.argtypes = [ctypes.c_uint64, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_int, u8p]
            lib.g4o_checksum.argtypes = [u8p, ctypes.c_size_t]
            lib.g4o_checksum.restype = ctypes.c_uint32
            _LIB = lib
        else:
            _LIB = False
    return _LIB or None


def name_hash(name: str) -> int:
    """FNV-1a over the name's UTF-8 bytes (FOG/scripts/fixture_prng.py:44-54)."""
    h = FNV_OFFSET
    for byte in name.encode("utf-8"):
        h = ((h ^ byte) * FNV_PRIME) & MASK64
    return h


def words(name: str, count: int, offset: int = 0) -> np.ndarray:
    """`count` u64 words for elements offset..offset+count (FOG/scripts/fixture_prng.py:57-67)."""
    index = np.arange(offset, offset + count, dtype=np.uint64)
    x = (np.uint64(name_hash(name)) ^ index) + GOLDEN
    x = (x ^ (x >> np.uint64(30))) * MIX_A
    x = (x ^ (x >> np.uint64(27))) * MIX_B
    return x ^ (x >> np.uint64(31))


def u01(w: np.ndarray) -> np.ndarray:
    return (w >> np.uint64(40)).astype(np.uint32).astype(np.float32) / np.float32(16777216.0)


def f32_to_bf16_bits(values) -> np.ndarray:
    """Round-half-to-even f32 -> bf16 bit patterns (finite inputs only)."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    rounding = np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))
    return ((bits + rounding) >> np.uint32(16)).astype(np.uint16)


def bf16_uniform(name: str, count: int, lo: float, hi: float) -> np.ndarray:
    u = u01(words(name, count))
    lo32, hi32 = np.float32(lo), np.float32(hi)
    return f32_to_bf16_bits(lo32 + (hi32 - lo32) * u)


def f32_uniform(name: str, count: int, lo: float, hi: float) -> np.ndarray:
    u = u01(words(name, count))
    lo32, hi32 = np.float32(lo), np.float32(hi)
    return lo32 + (hi32 - lo32) * u


def bf16_signs(name: str, count: int, scale: float = 1.0) -> np.ndarray:
    magnitude = f32_to_bf16_bits(np.array([abs(scale)], dtype=np.float32))[0]
    negative = words(name, count) >> np.uint64(63)
    return np.where(negative == 1, magnitude | np.uint16(0x8000), magnitude).astype(np.uint16)


def f8_banded(name: str, count: int, exp_min: int, exp_max: int, signed: bool = True) -> np.ndarray:
    """e4m3 code bytes whose exponent field lies in [exp_min, exp_max]."""
    assert 0 <= exp_min <= exp_max <= 14, f"{name}: exponent band {exp_min}..{exp_max} out of range"
    lib = _lib()
    if lib is not None and count >= (1 << 16):
        out = np.empty(count, dtype=np.uint8)
        lib.g4o_f8_banded(name_hash(name), count, exp_min, exp_max, int(signed),
                          out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)))
        return out
    w = words(name, count)
    span = exp_max - exp_min + 1
    exponent = (np.uint8(exp_min) + ((w >> np.uint64(32)) % np.uint64(span)).astype(np.uint8)).astype(np.uint8)
    mantissa = ((w >> np.uint64(56)) & np.uint64(0x7)).astype(np.uint8)
    sign = ((w >> np.uint64(63)).astype(np.uint8) << np.uint8(7)) if signed else np.uint8(0)
    return (sign | (exponent << np.uint8(3)) | mantissa).astype(np.uint8)


def f4_nibbles(name: str, count: int) -> np.ndarray:
    """`count` e2m1 codes packed two per byte, element 2i in the low nibble."""
    assert count % 2 == 0, f"{name}: f4 element count must be even, got {count}"
    lib = _lib()
    if lib is not None and count >= (1 << 16):
        out = np.empty(count // 2, dtype=np.uint8)
        lib.g4o_f4_nibbles(name_hash(name), count, out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)))
        return out
    codes = (words(name, count) >> np.uint64(60)).astype(np.uint8) & np.uint8(0xF)
    return (codes[0::2] | (codes[1::2] << np.uint8(4))).astype(np.uint8)


def checksum(storage: np.ndarray) -> int:
    """Position-weighted u32 checksum of a tensor's bytes (zero-padded to whole words)."""
    data = np.ascontiguousarray(storage).view(np.uint8).reshape(-1)
    lib = _lib()
    if lib is not None and data.size >= (1 << 20):
        return int(lib.g4o_checksum(data.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), data.size))
    padding = (-data.size) % 4
    if padding:
        data = np.concatenate([data, np.zeros(padding, dtype=np.uint8)])
    block = data.view(np.uint32)
    index = np.arange(block.size, dtype=np.uint32)
    return int((block * (index * np.uint32(2) + np.uint32(1))).sum(dtype=np.uint32)) & 0xFFFF_FFFF
