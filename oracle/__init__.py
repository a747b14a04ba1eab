"""CPU oracle for the Gemma-4 decode-layer ops: TEST INFRASTRUCTURE ONLY.

A restatement of the reference's CPU computation (its PyTorch fixture generator and the
grader's input synthesis) used to check the CUDA library. Only `tests/`,
`__graft_entry__.smoke()` and the CPU legs of `bench.py` may import it, and only as the
checker or the timed CPU baseline. The product path never routes through it: the CUDA
library has no CPU fallback.
"""
