"""TEST INFRASTRUCTURE ONLY -- CPU oracle for the Kalman Delta Network scan.

This package is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The shipped operators in
``kalman-delta-networks_b200/kdn_b200`` never import it and fail loudly when
the CUDA library is missing.

Parity status: pinned.  ``tests/golden/make_golden.py`` evaluates the
reference's own PyTorch oracles (``lit_gpt/kdn_ops/iso_kdn_naive.py`` and
``lit_gpt/kdn_ops/diag_kdn_naive.py``) on seeded inputs and commits their
outputs and gradients as fixtures; ``tests/test_oracle.py`` checks this
restatement against them.  The two gate frontends have no PyTorch oracle in
the reference: ``tests/golden/make_gate_golden.py`` runs the reference's own
Triton frontend kernels under Triton's CPU interpreter
(``iso_kdn_chunk.py:1059-1314``, ``diag_kdn_chunk.py:2218-2443``) and the
same test file pins ``iso_gate`` / ``diag_gate`` and their gradients to them.
"""

from .kdn_oracle import *  # noqa: F401,F403
