"""CPU oracle for the fused-step hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy float32, the two kernel families that the
reference compiler generates as Triton source:

* ``fp_chain_<N>`` flat / rows  (reference ``lib/Plan/TritonEmitter.cpp:14-65``,
  Python twin ``python/fusionpass/kernels.py:129-211``)
* ``fp_attention``              (reference ``lib/Plan/TritonEmitter.cpp:73-104``,
  Python twin ``python/fusionpass/kernels.py:58-89``)

It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / reference arm may import it.  The product path
(``fusionpass_b200``) never imports this package and has no CPU fallback.

Parity pin: every function here is checked against golden vectors produced by
running the reference's own Triton kernels under ``TRITON_INTERPRET=1``
(``tests/golden/make_golden.py`` writes them; ``tests/test_oracle_golden.py``
checks them).
"""

from .chain import chain_eval, chain_flat, chain_rows, body_to_program  # noqa: F401
from .attention import attention_fwd  # noqa: F401
