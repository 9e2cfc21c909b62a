"""CPU restatement of torchcst's radius cell-mass Linear training step.

TEST INFRASTRUCTURE ONLY. Nothing in the ``torchcst_b200`` package imports,
links or calls this package. Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm use it, and only as the checker or
as the timed CPU stand-in for the reference's own factored backend.

Parity pin: the restatement is checked against golden vectors produced by the
reference package itself (``tests/golden/make_golden.py`` imports torchcst and
writes ``tests/golden/*.npz``); see ``tests/test_oracle_golden.py``.
"""

from .cst_oracle import *  # noqa: F401,F403
