"""CPU oracle for the paged-KV hot path.  TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the algorithms of the reference engine
(mini-engine, ``mini_engine/kernels`` and ``mini_engine/engine/batch.py``)
for every operation that the CUDA library in ``myvllm_mini_engine_b200``
implements.  Each function cites the reference file:line it follows.

Who may use it: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` -- as the checker
or as the timed CPU baseline.  The product package never imports it and has
no CPU fallback.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own torch
paths on the seeded cases of ``tests/golden/cases.py`` and stores their
outputs; ``tests/test_oracle_golden.py`` checks this oracle against those
fixtures and against the literal golden vectors of the reference tests.

Arithmetic: byte/index work (KV writes, copy-on-write, metadata) is numpy or
plain Python and bit-exact; attention is torch fp32 on the CPU, exactly as the
reference's fallback path computes it.
"""
