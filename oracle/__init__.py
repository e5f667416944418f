"""CPU oracle for the GRINQH quantized-linear hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this module;
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / reference
arm of ``bench.py`` may use it, and only as the checker or as the timed CPU
baseline, never as the thing measured for the GPU path.

The restatement is pinned against the reference's own kernels: the fixtures in
``tests/golden/`` were produced by the reference's Triton kernels
(``_pack_kernel_uint32``, ``grinqh_gemv_uint32_packed``,
``grinqh_gemv_uint32_packed_batch_union``) run under the Triton CPU interpreter
and by its eager dense path, see ``tests/golden/make_golden.py``.
"""
from .grinqh_oracle import *  # noqa: F401,F403
