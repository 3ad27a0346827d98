"""CPU oracle for the GSQ / GPTQ / RCO hot path. TEST INFRASTRUCTURE ONLY.

Nothing in the product package imports this directory. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and its
``--impl reference`` arm) may import it, and only as the checker or the timed CPU
baseline, never as a code path of the CUDA product.

Each function restates the reference algorithm of egesabanci/gsq-rco-mlx in plain
numpy (or C, ``oracle/dp.c``) and cites the reference file:line it follows.
Pinning: the pieces whose reference code is numpy (GPTQ, RTN, grid, schedules,
inits, DP, RCO manifold/loop) are checked against golden vectors produced by the
reference itself (``tests/golden/make_golden.py``). The MLX-only pieces (Gumbel
soft weight, stage losses, Lion) are checked against the reference test oracle
``tests/oracles.py`` (2-bit full grid, Lion) through the same golden file, and
against finite differences for the local-shift gradients.
"""
