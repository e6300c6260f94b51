"""CPU oracle and eager baseline for the Block AttnRes operator.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
(as the checker) and ``bench.py``'s CPU-baseline leg. The product path
(``switchyard``) never imports it.
"""
