"""TEST INFRASTRUCTURE ONLY: the CPU oracle for the Cheetah decoder hot path.

A C++ restatement (`ref_cpu.cpp`) of the reference native backend
(`src/chat/native/ops.rs`, `src/chat/registrations/qwen2.rs`,
`src/chat/precision/{q8,q4}.rs`), wrapped with ctypes. Used only by
`tests/`, `__graft_entry__.smoke()` and bench.py's CPU-baseline leg, as the
checker and the timed CPU baseline. The product library never imports it.
"""

from .ref import *  # noqa: F401,F403
