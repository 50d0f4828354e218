"""CPU oracle for the paged-KV hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` legs may import this package, and only as the checker
or as the timed CPU baseline. The product package (``mi_b200``) never imports
it: the product path is the CUDA library, and it fails loudly when that
library is missing.

Parity status: pinned. ``tests/golden/`` holds fixtures produced by running
the reference (cartesia-ai/minimal-inference ``model.py`` / ``scheduler.py``)
on CPU; ``tests/test_oracle_golden.py`` checks this oracle against them.
"""
