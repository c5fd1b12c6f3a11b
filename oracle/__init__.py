"""CPU oracle for the RUNE energy/force/virial path — TEST INFRASTRUCTURE ONLY.

This package restates, in float64 numpy, the arithmetic of the RUNE reference PyTorch code
(Jonsnow-willow/Rune, ``rune/mobius/*.py`` and ``rune/nep/*.py``) for the hot path that the
CUDA engine in ``rune_b200`` implements: the periodic neighbour list, the NEP/Möbius radial and
angular descriptors, the NEP per-element network, the Möbius Local / MP / EQ networks, ZBL, and
the analytic force and virial contraction. Each function cites the reference file:line it
follows.

Parity status: pinned. ``tests/test_oracle_golden.py`` checks every function here against the
golden vectors in ``tests/golden/``, which ``tests/golden/make_golden.py`` produced by running
the reference implementation itself.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import this package, and only as the checker or the timed CPU
baseline. The product (``rune_b200``) never imports it.
"""
