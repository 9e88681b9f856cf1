"""CPU oracle for the MRSA route-layer / SWA-layer forward path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
module; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of
``bench.py`` (``cpu_baseline`` and ``--impl reference``) use it, and only as
the checker or as the timed CPU baseline.  It is a restatement in plain torch
(CPU, fp32 math, bf16 storage where the reference stores bf16) of the
reference's own PyTorch path; every function names the reference file:line it
follows.  It is pinned against outputs of the reference itself by the golden
fixtures under ``tests/golden/`` (see ``tests/golden/make_golden.py``).
"""

from .route_layer import *  # noqa: F401,F403
from . import token_ops  # noqa: F401
