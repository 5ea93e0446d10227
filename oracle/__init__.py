"""Test infrastructure only: the CPU restatement of the reference LTC solver.

Nothing in the product (the ``ltc-cuda_b200`` package, the shared library)
imports this package; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, as a
checker or as the timed CPU baseline.
"""
