"""g4b200: B200 (sm_100a) kernels for the Gemma-4-12B decoder-layer ops behind a C ABI.

`g4b200.ops` mirrors the reference's `furiosa-opt-gemma4-12B/src/ops.rs` entry points;
`g4b200._abi` is the ctypes binding of `libg4b200.so` (include/g4b200.h).
"""

from ._abi import G4Error, LIB_PATH, LibraryMissing, lib  # noqa: F401

__all__ = ["G4Error", "LIB_PATH", "LibraryMissing", "lib"]
