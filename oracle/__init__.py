"""CPU oracle for the W4A8 integer decode path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy and plain C, the integer law of the
reference model (coreyhahn/fable5_llm ``ref/w4a8_ref.py``,
``ref/fixedpoint.py``, ``ref/layer_fixed.py``).  It exists to CHECK the CUDA
implementation in ``fable5_llm_b200``; it is never the thing measured or
shipped.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.

Parity of the oracle itself is pinned by the committed fixtures under
``tests/golden/`` (generated from the unmodified reference by
``tests/golden/gen_golden.py``).
"""
from .oracle import *  # noqa: F401,F403
