"""CPU oracle for the B200 backend's parity tests -- TEST INFRASTRUCTURE ONLY.

Nothing in the shipped backend imports this package.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arms
may import it, and only as the checker (or as the timed host baseline), never
as a stand-in for a GPU result.

Contents (each function cites the reference file:line it restates):

* :mod:`oracle.tf32`   -- the 3xTF32 arithmetic model (tf32_emitter.py:22-96).
* :mod:`oracle.refs`   -- the reference's float64 NumPy equations per kernel
  family (tools/research_cases.py:74-103, tests/performance/generators/suite.py:192-234).
* :mod:`oracle.sexp`   -- the selective subnormal-preserving exponential
  (compile.py:2953-2965) as a CPU model with its error bound.

Parity is pinned: ``tests/test_oracle.py`` checks these functions against the
bundled expected outputs (``tests/golden/cases/*/expected.npz``) and against
outputs of the reference's own ``tf32_emitter`` (``tests/golden/tf32``).
"""
