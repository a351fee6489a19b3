"""CPU oracle for the paged-attention hot path.  TEST INFRASTRUCTURE ONLY.

Imported by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` as the checker; the product package never imports it.
"""
