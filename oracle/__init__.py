"""CPU oracle for the TAGI moment hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch on the CPU, the moment equations that
triton-tagi's Triton kernels and layer classes compute. It exists for three
callers only:

* ``tests/``               — the checker every CUDA result is compared with;
* ``__graft_entry__.smoke`` — one small parity check on ``cuda:0``;
* ``bench.py``             — the timed CPU baseline (``cpu_baseline`` and
                             ``--impl reference``).

The product path (``triton-tagi_b200/triton_tagi``) never imports it: the
CUDA library is the only implementation there, and it fails loudly when the
library cannot be loaded.

Parity pin: every function here is checked against golden vectors produced by
running the reference implementation itself (its Triton kernels under
``TRITON_INTERPRET=1`` on the CPU) — see ``tests/golden/make_golden.py`` and
``tests/test_oracle_golden.py``.
"""

from . import moments, net  # noqa: F401
