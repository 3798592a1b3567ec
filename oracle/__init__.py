"""CPU oracle for the Muon update hot path -- TEST INFRASTRUCTURE ONLY.

This package is a NumPy restatement of the reference's Muon update
(RhizomeResearch/rollfast, ``src/rollfast/optim/muon.py``,
``src/rollfast/optim/orthogonalization.py``, ``src/rollfast/utils.py``,
``src/rollfast/optim/dimension_numbers.py``, ``src/rollfast/optim/adam.py``).
Every function cites the reference file:line it follows.

It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s ``cpu_baseline`` / ``--impl reference`` legs may import it.
The CUDA path in ``rollfast_b200`` never routes through this package.

Pinning: the reference is pure JAX/Optax, which is not installable in this
image (no jax/jaxlib/optax wheels, no network), so the reference itself cannot
be run to produce fixtures.  The oracle is pinned instead against every
known-answer test the reference's own test-suite holds for this path (see
``tests/test_oracle_known_answers.py``); the numerics that JAX leaves
unpinned (matmul summation order, fp32 ``pow``) are computed here in float32
("reference-equivalent") and float64 ("truth").
"""

from .muon_np import *  # noqa: F401,F403
