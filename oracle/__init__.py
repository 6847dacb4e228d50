"""CPU oracle for the cormorant_b200 kernels — TEST INFRASTRUCTURE ONLY.

This package restates, in plain numpy (and Python integers where a value
exceeds 64 bits), the fixed-point arithmetic of the reference simulator
(phoenix367/cormorant, ``inference-scheduler/src``) and of the register-level
kernel emulators of its test suite (``inference-scheduler/test/host_emu.py``,
``kernels/rowops_rtl/tb/verilator/rowops_ref.h``).  Every function cites the
reference file:line it follows.

Who may use it: ``tests/`` (as the checker), ``__graft_entry__.smoke()`` (as
the checker) and ``bench.py`` (the ``cpu_baseline`` leg and ``--impl
reference``).  The product package ``cormorant_b200`` never imports it: the
GPU path has no CPU fallback.

Pinning: ``tests/test_oracle_golden.py`` checks these functions against the
reference's own register-level fixtures (``hw/test_data``, converted to
``tests/golden/hw_*.npz`` by ``tests/golden/make_golden.py``) and against
outputs of the reference Python simulator run in the build container
(``tests/golden/sim_*.npz``, same script).
"""
