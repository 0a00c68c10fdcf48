"""CPU oracle for the MPQ per-layer quantization solve.

TEST INFRASTRUCTURE ONLY.  This package is a plain numpy (float32) restatement of
the reference algorithm (poseidonchan/MPQ, ``mpq/solver.py``, ``mpq/linear.py``,
``mpq/priors/*``, ``mpq/polish/*``, ``mpq/adapters/*``).  Every function cites the
reference ``file:line`` it follows.

It exists to CHECK the CUDA product, never to BE it: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it.  The product package ``mpq_b200`` never imports it and
fails loudly when its CUDA library is missing.

Pinning: ``tests/golden/*.npz`` hold input/output vectors produced by importing the
reference itself (generator: ``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py``
checks this restatement against them.
"""
