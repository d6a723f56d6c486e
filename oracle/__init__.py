"""CPU oracle for the hot-path ops -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference programs that
Yihuace/tile-ascendnpu-ops checks its operators against (the ``ref_program``
methods of ``examples/TileOPs/tests/ops/test_*.py`` and the ``golden_*``
functions beside its kernels).  Each function names the reference file:line
it follows.

It exists to CHECK the CUDA kernels, never to run in their place: only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import it.  The ``tileops`` package does not import it and has
no CPU fallback.

Parity pinning: ``tests/golden/make_golden.py`` executes the reference's own
ref programs / goldens (from the reference checkout, in the build container)
on seeded inputs and commits the results as fixtures; ``tests/test_oracle.py``
checks every function here against those fixtures.  GDN prefill has no
reference test; its oracle is pinned to the reference's sequential golden
(examples/gdn_prefill/probe/gdn_prefill_probe.py:60-77) and cross-checked
against flash-linear-attention's CPU reference recurrence (the probe's
ref_api library).
"""

from oracle import reference

__all__ = ["reference"]
